// esa_layer.cu -- the ESA layer core behind esa_layer_fwd / esa_layer_bwd:
// gated scan of the qgv logits, then the RMS readout (forward), or the
// readout backward, then the reverse gated scan (backward).
//
// The two steps are separate launches on the caller's stream: the scan
// kernels (esa_strip.cuh) make their parallelism from channel strips that
// sweep the whole time axis, the readout needs every channel of a step, so a
// single kernel would have to chain tiles of all channels along the time
// axis.  That fused form was built and measured on B200 (row tiles of a few
// steps x all channels, decoupled look-back between tiles): on the
// [16, 2048, 768] fp16 training layer it took 148 us forward / 282 us
// backward against 104 / 154 us for these two launches, its tiles waiting on
// the look-back chain; it is not kept.
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"

namespace esa {
namespace {

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int check_layer_dims(int64_t nb, int64_t T, int64_t C) {
    if (nb < 0 || T < 0 || C <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "layer core needs nb, T >= 0 and C > 0");
    if (nb > 0x7fffffffLL || T > 0x7fffffffLL || C > 0x7fffffffLL)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "dimension exceeds 2^31 - 1");
    return ESA_OK;
}

int widest(int a, int b) { return dtype_size(a) >= dtype_size(b) ? dtype_size(a) : dtype_size(b); }

}  // namespace

// The gated scan's workspace, plus dE between the readout backward and the
// reverse scan.
size_t layer_workspace_bytes(int64_t nb, int64_t T, int64_t C, int qdt, int edt, int ydt) {
    if (nb < 0 || T < 0 || C <= 0 || dtype_size(qdt) == 0 || dtype_size(edt) == 0 || dtype_size(ydt) == 0) return 0;
    const size_t scan = scan_workspace_bytes(nb, T, C, widest(qdt, edt), 16);
    return align256((size_t)(nb * T * C) * dtype_size(edt)) + scan;
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
    const size_t de_bytes = align256((size_t)(nb * T * C) * ees);
    if (ws == nullptr || ws_bytes < de_bytes || (reinterpret_cast<uintptr_t>(ws) & 255u))
        return set_error(ESA_ERR_WORKSPACE, "layer backward workspace smaller than esa_layer_workspace_bytes()");
    char* dE = static_cast<char*>(ws);
    if (int rc = readout_bwd(dy, C, dydt, q, qrs, qdt, E, C, edt, rstd, dq, dqrs, qdt, dE, C, edt, nb * T, C, eps, s))
        return rc;
    return gated_scan_bwd(g, v, qrs, qdt, E, dE, edt, dg, dv, dqrs, qdt, nb, T, C, gmin, gmax, 1, 16, e0, de0,
                          dE + de_bytes, ws_bytes - de_bytes, s);
}

}  // namespace esa
