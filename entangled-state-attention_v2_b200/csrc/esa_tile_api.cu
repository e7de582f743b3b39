// esa_tile_api.cu -- the fused ESA layer core (gated scan + RMS readout in one
// kernel per direction) and the row-tile path of the bare gated scans.
//
// Planning: a tile is LT steps x all C channels of one batch row; C splits
// into NWC = C / (32 V) consumer warps of 32 V channels (V = 2 or 4 channels
// per lane, at most 12 warps).  Each candidate (V, LT) in the order
// (2, 16), (2, 8), (4, 8) is taken if every staged element type gives a
// 4-, 8- or 16-byte lane vector and at least two stages of the ring fit in
// shared memory.  Shapes or dtype mixes that no candidate covers run the
// two-kernel form (gated scan, then the readout) through the same entry
// points, so a caller sees the same results either way.
#include <cstring>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"
#include "esa_tile_launch.cuh"

namespace esa {
namespace {

constexpr int kMaxStages = TileSmem::MAX_STAGES;
// dynamic shared memory the ring may use (the kernel's tail -- barriers,
// tile ids, readout partials -- takes under 2 KB on top)
constexpr int kRingBudget = 220 * 1024;
// ring depth: two stages are one tile in flight while one is consumed; a
// third lets the producer run ahead of a tile waiting on its look-back
constexpr int kStagesWanted = 3;

struct TilePlan {
    bool ok = false;
    int v = 0, lt = 0, nwc = 0, wb = 0, nstage = 0, stage_bytes = 0;
    int arr_off[5] = {0, 0, 0, 0, 0};
    int arr_rows[5] = {0, 0, 0, 0, 0};
    int64_t G = 0, ntiles = 0;
    size_t flags_bytes = 0, agg_bytes = 0, ws_bytes = 0;
};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

bool is16(int dt) { return dt == ESA_DTYPE_F16 || dt == ESA_DTYPE_BF16; }

// element size of staged array i (g, v, q, E, dY)
int arr_es(bool rev, bool ro, int i, int tr, int te, int ty) {
    if (i < 3) return dtype_size(tr);
    if (i == 3) return dtype_size(te);
    return dtype_size(ro ? ty : te);
}

TilePlan tile_plan(bool rev, bool ro, int tr, int te, int ty, int64_t nb, int64_t T, int64_t C) {
    TilePlan p;
    // the instantiated dtype mixes (esa_tile_*.cu)
    const bool same16 = is16(te) && tr == te && (!ro || ty == te);
    const bool all32 = tr == ESA_DTYPE_F32 && te == ESA_DTYPE_F32 && (!ro || ty == ESA_DTYPE_F32);
    const bool f32_16 = tr == ESA_DTYPE_F32 && is16(te) && (!ro || ty == ESA_DTYPE_F32);
    if (!(same16 || all32 || f32_16)) return p;
    if (nb <= 0 || T <= 0 || C <= 0 || C > 4096) return p;
    const int narr = rev ? 5 : 3;
    const int cands[3][2] = {{2, 16}, {2, 8}, {4, 8}};
    for (const auto& cand : cands) {
        const int v = cand[0], lt = cand[1];
        const int cw = 32 * v;
        if (C % cw != 0) continue;
        const int nwc = (int)(C / cw);
        if (nwc > TileSmem::MAX_WARPS) continue;
        bool vec_ok = true;
        for (int i = 0; i < narr; ++i) {
            if (i == 2 && !ro) continue;
            const int bytes = v * arr_es(rev, ro, i, tr, te, ty);
            if (bytes != 4 && bytes != 8 && bytes != 16) vec_ok = false;
        }
        if (ro && !rev) {
            const int bytes = v * dtype_size(ty);
            if (bytes != 4 && bytes != 8 && bytes != 16) vec_ok = false;
        }
        if (!vec_ok) continue;
        // TMA box: the widest multiple of the warp slice that divides C and
        // stays within 256 elements
        int wb = cw;
        for (int k = nwc; k >= 1; --k) {
            if (nwc % k == 0 && cw * k <= 256) {
                wb = cw * k;
                break;
            }
        }
        int off = 0;
        for (int i = 0; i < narr; ++i) {
            p.arr_off[i] = off;
            if (i == 2 && !ro) {
                p.arr_rows[i] = 0;
                continue;
            }
            const int rows = (rev && i == 3) ? lt + 1 : lt;
            p.arr_rows[i] = rows;
            off += rows * (int)C * arr_es(rev, ro, i, tr, te, ty);  // a multiple of 128 bytes
        }
        int ns = kRingBudget / off;
        if (ns < 2) continue;
        if (ns > kStagesWanted) ns = kStagesWanted;
        if (ns > kMaxStages) ns = kMaxStages;
        p.v = v;
        p.lt = lt;
        p.nwc = nwc;
        p.wb = wb;
        p.nstage = ns;
        p.stage_bytes = off;
        p.G = (T + lt - 1) / lt;
        p.ntiles = nb * p.G;
        if (p.ntiles >= (int64_t)0x7fffffff) return TilePlan{};
        p.flags_bytes = align256((size_t)p.ntiles * nwc * sizeof(unsigned));
        p.agg_bytes = align256((size_t)p.ntiles * C * sizeof(float));
        p.ws_bytes = 256 + p.flags_bytes + 3 * p.agg_bytes;
        p.ok = true;
        return p;
    }
    return p;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Fills the launch description shared by every kind; the caller sets the
// outputs and the staged inputs.
int tile_setup(const TilePlan& p, TileLaunch& L, int64_t nb, int64_t T, int64_t C, double gmin, double gmax,
               double eps, void* ws, cudaStream_t s) {
    memset(&L, 0, sizeof(L));
    TileArgs& a = L.a;
    a.nb = nb;
    a.T = T;
    a.C = C;
    a.G = p.G;
    a.ntiles = p.ntiles;
    a.nwc = p.nwc;
    a.wb = p.wb;
    a.nstage = p.nstage;
    a.stage_bytes = p.stage_bytes;
    for (int i = 0; i < 5; ++i) {
        a.arr_off[i] = p.arr_off[i];
        a.arr_rows[i] = p.arr_rows[i];
    }
    a.gmin = gmin;
    a.span = gmax - gmin;
    a.eps = eps;
    int dev = 0;
    cudaGetDevice(&dev);
    a.status = status_ptr(dev);
    if (a.status == nullptr) return set_error(ESA_ERR_CUDA, "cannot resolve the device status word");
    char* w = static_cast<char*>(ws);
    a.ticket = reinterpret_cast<unsigned*>(w);
    a.abort_flag = a.ticket + 1;
    a.flags = reinterpret_cast<unsigned*>(w + 256);
    a.agg_a = reinterpret_cast<float*>(w + 256 + p.flags_bytes);
    a.agg_b = reinterpret_cast<float*>(w + 256 + p.flags_bytes + p.agg_bytes);
    a.pref = reinterpret_cast<float*>(w + 256 + p.flags_bytes + 2 * p.agg_bytes);
    L.stream = s;
    // ticket, abort flag and every look-back flag start at zero
    const cudaError_t e = cudaMemsetAsync(ws, 0, 256 + p.flags_bytes, s);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("tile flags clear: ") + cudaGetErrorString(e));
    return ESA_OK;
}

bool ws_fits(const TilePlan& p, const void* ws, size_t ws_bytes) {
    return ws != nullptr && (reinterpret_cast<uintptr_t>(ws) & 255u) == 0 && ws_bytes >= p.ws_bytes;
}

int check_layer_dims(int64_t nb, int64_t T, int64_t C) {
    if (nb < 0 || T < 0 || C <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "layer core needs nb, T >= 0 and C > 0");
    if (nb > 0x7fffffffLL || T > 0x7fffffffLL || C > 0x7fffffffLL)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "dimension exceeds 2^31 - 1");
    return ESA_OK;
}

int widest(int a, int b) { return dtype_size(a) >= dtype_size(b) ? dtype_size(a) : dtype_size(b); }

}  // namespace

size_t layer_workspace_bytes(int64_t nb, int64_t T, int64_t C, int qdt, int edt, int ydt) {
    if (nb < 0 || T < 0 || C <= 0 || dtype_size(qdt) == 0 || dtype_size(edt) == 0 || dtype_size(ydt) == 0) return 0;
    const TilePlan f = tile_plan(false, true, qdt, edt, ydt, nb, T, C);
    const TilePlan r = tile_plan(true, true, qdt, edt, ydt, nb, T, C);
    size_t need = 256;
    if (f.ok && f.ws_bytes > need) need = f.ws_bytes;
    if (r.ok && r.ws_bytes > need) need = r.ws_bytes;
    if (!f.ok || !r.ok) {
        // the two-kernel form: the gated scan's workspace, plus dE between the
        // readout backward and the reverse scan
        const size_t scan = scan_workspace_bytes(nb, T, C, widest(qdt, edt), 16);
        const size_t fb = align256((size_t)(nb * T * C) * dtype_size(edt)) + scan;
        if (fb > need) need = fb;
    }
    return need;
}

int layer_fwd(const void* qgv, int64_t qrs, int qdt, void* E, int edt, void* y, int ydt, void* rstd, int64_t nb,
              int64_t T, int64_t C, double gmin, double gmax, double eps, const void* e0, void* e_last, void* ws,
              size_t ws_bytes, cudaStream_t s) {
    if (int rc = check_layer_dims(nb, T, C)) return rc;
    const int qes = dtype_size(qdt), ees = dtype_size(edt), yes = dtype_size(ydt);
    if (qes == 0 || ees == 0 || yes == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code");
    if (qrs < 3 * C) return set_error(ESA_ERR_INVALID_ARGUMENT, "qgv row stride smaller than 3*C");
    if (nb * T == 0) return ESA_OK;
    if (!qgv || !E || !y || !rstd) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    const char* q = static_cast<const char*>(qgv);
    const char* g = q + C * qes;
    const char* v = q + 2 * C * qes;
    const TilePlan p = tile_plan(false, true, qdt, edt, ydt, nb, T, C);
    const bool aligned = al16(q) && (qrs * qes) % 16 == 0 && (C * qes) % 16 == 0 && al16(E) && al16(y) &&
                         (C * ees) % 16 == 0 && (C * yes) % 16 == 0;
    if (p.ok && aligned && ws_fits(p, ws, ws_bytes)) {
        TileLaunch L;
        if (int rc = tile_setup(p, L, nb, T, C, gmin, gmax, eps, ws, s)) return rc;
        L.a.out0 = static_cast<char*>(E);
        L.a.o0rs = C;
        L.a.out1 = static_cast<char*>(y);
        L.a.o1rs = C;
        L.a.rstd = rstd;
        L.a.e0 = e0;
        L.a.e_last = e_last;
        const char* ins[3] = {g, v, q};
        for (int i = 0; i < 3; ++i) {
            L.in[i] = ins[i];
            L.in_rs[i] = qrs;
            L.in_dt[i] = qdt;
        }
        note_scan_path(ESA_PATH_ROWTILE);
        return tile_launch_fwd_ro(qdt, edt, ydt, p.v, p.lt, L);
    }
    // two kernels: the gated scan writes E, the readout reads it back
    if (int rc = gated_scan_fwd(g, v, qrs, qdt, E, edt, nb, T, C, gmin, gmax, 1, 16, e0, e_last, ws, ws_bytes, s))
        return rc;
    return readout_fwd(q, qrs, qdt, E, C, edt, y, C, ydt, rstd, nb * T, C, eps, s);
}

int layer_bwd(const void* dy, int dydt, const void* qgv, int64_t qrs, int qdt, const void* E, int edt,
              const void* rstd, void* dqgv, int64_t dqrs, int64_t nb, int64_t T, int64_t C, double gmin, double gmax,
              double eps, const void* e0, void* de0, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (int rc = check_layer_dims(nb, T, C)) return rc;
    const int qes = dtype_size(qdt), ees = dtype_size(edt), dyes = dtype_size(dydt);
    if (qes == 0 || ees == 0 || dyes == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code");
    if (qrs < 3 * C || dqrs < 3 * C) return set_error(ESA_ERR_INVALID_ARGUMENT, "qgv row stride smaller than 3*C");
    if (nb * T == 0) return ESA_OK;
    if (!dy || !qgv || !E || !rstd || !dqgv) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    const char* q = static_cast<const char*>(qgv);
    const char* g = q + C * qes;
    const char* v = q + 2 * C * qes;
    char* dq = static_cast<char*>(dqgv);
    char* dg = dq + C * qes;
    char* dv = dq + 2 * C * qes;
    const TilePlan p = tile_plan(true, true, qdt, edt, dydt, nb, T, C);
    const bool aligned = al16(q) && (qrs * qes) % 16 == 0 && (C * qes) % 16 == 0 && al16(dq) &&
                         (dqrs * qes) % 16 == 0 && al16(E) && (C * ees) % 16 == 0 && al16(dy) && (C * dyes) % 16 == 0;
    if (p.ok && aligned && ws_fits(p, ws, ws_bytes)) {
        TileLaunch L;
        if (int rc = tile_setup(p, L, nb, T, C, gmin, gmax, eps, ws, s)) return rc;
        L.a.out0 = dg;
        L.a.o0rs = dqrs;
        L.a.out1 = dv;
        L.a.o1rs = dqrs;
        L.a.out2 = dq;
        L.a.o2rs = dqrs;
        L.a.rstd = const_cast<void*>(rstd);
        L.a.e0 = e0;
        L.a.e_last = de0;
        const void* ins[5] = {g, v, q, E, dy};
        const int64_t rss[5] = {qrs, qrs, qrs, C, C};
        const int dts[5] = {qdt, qdt, qdt, edt, dydt};
        for (int i = 0; i < 5; ++i) {
            L.in[i] = ins[i];
            L.in_rs[i] = rss[i];
            L.in_dt[i] = dts[i];
        }
        note_scan_path(ESA_PATH_ROWTILE);
        return tile_launch_rev_ro(qdt, edt, dydt, p.v, p.lt, L);
    }
    // two kernels: the readout backward writes dq and dE, the reverse scan
    // reads dE back
    const size_t de_bytes = align256((size_t)(nb * T * C) * ees);
    if (ws == nullptr || ws_bytes < de_bytes || (reinterpret_cast<uintptr_t>(ws) & 255u))
        return set_error(ESA_ERR_WORKSPACE, "layer backward workspace smaller than esa_layer_workspace_bytes()");
    char* dE = static_cast<char*>(ws);
    if (int rc = readout_bwd(dy, C, dydt, q, qrs, qdt, E, C, edt, rstd, dq, dqrs, qdt, dE, C, edt, nb * T, C, eps, s))
        return rc;
    return gated_scan_bwd(g, v, qrs, qdt, E, dE, edt, dg, dv, dqrs, qdt, nb, T, C, gmin, gmax, 1, 16, e0, de0,
                          dE + de_bytes, ws_bytes - de_bytes, s);
}

// The bare gated scans on the row-tile kernel (no readout): *taken = false
// when the plan, the alignment or the workspace does not allow it, or when
// the problem has fewer tiles than SMs (short single sequences keep the
// other kernels, which split the channels as well as the time axis).
int tile_gated_fwd(const ScanCall& c, bool* taken) {
    *taken = false;
    const KArgs& k = c.a;
    if (!(k.round_ab || c.te == ESA_DTYPE_F32)) return ESA_OK;
    const TilePlan p = tile_plan(false, false, c.tin, c.te, c.te, k.nb, k.T, k.hd);
    if (!p.ok || !ws_fits(p, c.ws, c.ws_bytes) || !c.bulk_ok) return ESA_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    if (p.ntiles < device_sm_count(dev)) return ESA_OK;
    TileLaunch L;
    if (int rc = tile_setup(p, L, k.nb, k.T, k.hd, k.gmin, k.gmin + k.span, 0.0, c.ws, c.stream)) return rc;
    L.a.out0 = k.out[0].p;
    L.a.o0rs = k.out[0].rs;
    L.a.e0 = k.e0;
    L.a.e_last = k.e_last;
    for (int i = 0; i < 2; ++i) {
        L.in[i] = k.in[i].p;
        L.in_rs[i] = k.in[i].rs;
        L.in_dt[i] = c.tin;
    }
    *taken = true;
    note_scan_path(ESA_PATH_ROWTILE);
    return tile_launch_fwd_plain(c.tin, c.te, c.te, p.v, p.lt, L);
}

int tile_gated_bwd(const ScanCall& c, bool* taken) {
    *taken = false;
    const KArgs& k = c.a;
    if (!(k.round_ab || c.te == ESA_DTYPE_F32)) return ESA_OK;
    const TilePlan p = tile_plan(true, false, c.tin, c.te, c.te, k.nb, k.T, k.hd);
    if (!p.ok || !ws_fits(p, c.ws, c.ws_bytes) || !c.bulk_ok) return ESA_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    if (p.ntiles < device_sm_count(dev)) return ESA_OK;
    TileLaunch L;
    if (int rc = tile_setup(p, L, k.nb, k.T, k.hd, k.gmin, k.gmin + k.span, 0.0, c.ws, c.stream)) return rc;
    L.a.out0 = k.out[0].p;
    L.a.o0rs = k.out[0].rs;
    L.a.out1 = k.out[1].p;
    L.a.o1rs = k.out[1].rs;
    L.a.e0 = k.e0;
    L.a.e_last = k.e_last;
    // staged: g, v, (no q), E, dE
    const int order[4] = {0, 1, 3, 4};
    for (int j = 0; j < 4; ++j) {
        const int i = order[j];
        L.in[i] = k.in[j].p;
        L.in_rs[i] = k.in[j].rs;
        L.in_dt[i] = j < 2 ? c.tin : c.te;
    }
    *taken = true;
    note_scan_path(ESA_PATH_ROWTILE);
    return tile_launch_rev_plain(c.tin, c.te, c.te, p.v, p.lt, L);
}

size_t tile_gated_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int dtype) {
    // the dtype mixes whose widest element type is `dtype`
    int mixes[3][2] = {{dtype, dtype}, {-1, -1}, {-1, -1}};
    if (dtype == ESA_DTYPE_F32) {
        mixes[1][0] = mixes[2][0] = ESA_DTYPE_F32;
        mixes[1][1] = ESA_DTYPE_F16;
        mixes[2][1] = ESA_DTYPE_BF16;
    }
    size_t need = 0;
    for (const auto& m : mixes) {
        if (m[0] < 0) continue;
        for (int rev = 0; rev < 2; ++rev) {
            const TilePlan p = tile_plan(rev != 0, false, m[0], m[1], m[1], nb, T, hd);
            if (p.ok && p.ws_bytes > need) need = p.ws_bytes;
        }
    }
    return need;
}

}  // namespace esa
