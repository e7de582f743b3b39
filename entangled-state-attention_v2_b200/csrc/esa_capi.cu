// esa_capi.cu -- the extern "C" entry points declared in include/esa_b200.h.
//
// Thin wrappers: argument checks that need no device work, the thread-local
// last-error string, and dispatch to the kernels' host launchers.
#include <mutex>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"

namespace esa {

static thread_local std::string t_last_error;

int set_error(int code, const std::string& msg) {
    t_last_error = msg;
    return code;
}

void clear_error() { t_last_error.clear(); }

static thread_local int t_last_path = 0;
void note_scan_path(int path) { t_last_path = path; }
int last_scan_path() { return t_last_path; }

int device_sm_count(int device) {
    static int cache[64] = {0};
    static std::mutex mu;
    if (device < 0 || device >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
            n = 148;
        cache[device] = n;
    }
    return cache[device];
}

}  // namespace esa

using namespace esa;

// the library is built with hidden visibility; only the C ABI is exported
#define ESA_EXPORT __attribute__((visibility("default")))

extern "C" {

ESA_EXPORT int esa_abi_version(void) { return ESA_ABI_VERSION; }

ESA_EXPORT const char* esa_last_error(void) { return t_last_error.c_str(); }

ESA_EXPORT int esa_scan_last_path(void) { return last_scan_path(); }

ESA_EXPORT int esa_cross_entropy_fwd(const void* logits, int64_t row_stride, int dtype, const int64_t* targets,
                                     int64_t ignore_index, float* lse, float* loss, int64_t rows, int64_t V,
                                     void* stream) {
    clear_error();
    return cross_entropy_fwd(logits, row_stride, dtype, targets, ignore_index, lse, loss, rows, V,
                             static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_cross_entropy_bwd(const void* logits, int64_t row_stride, int dtype, const int64_t* targets,
                                     int64_t ignore_index, const float* lse, const float* grad_rows, void* dlogits,
                                     int64_t dlogits_row_stride, int64_t rows, int64_t V, void* stream) {
    clear_error();
    return cross_entropy_bwd(logits, row_stride, dtype, targets, ignore_index, lse, grad_rows, dlogits,
                             dlogits_row_stride, rows, V, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_readout_fwd(const void* q, int64_t q_row_stride, int q_dtype, const void* E,
                               int64_t e_row_stride, int e_dtype, void* y, int64_t y_row_stride,
                               int y_dtype, void* rstd, int64_t rows, int64_t C, double eps,
                               void* stream) {
    clear_error();
    return readout_fwd(q, q_row_stride, q_dtype, E, e_row_stride, e_dtype, y, y_row_stride, y_dtype, rstd,
                       rows, C, eps, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_readout_bwd(const void* dy, int64_t dy_row_stride, int dy_dtype, const void* q,
                               int64_t q_row_stride, int q_dtype, const void* E, int64_t e_row_stride,
                               int e_dtype, const void* rstd, void* dq, int64_t dq_row_stride,
                               int dq_dtype, void* dE, int64_t de_row_stride, int de_dtype, int64_t rows,
                               int64_t C, double eps, void* stream) {
    clear_error();
    return readout_bwd(dy, dy_row_stride, dy_dtype, q, q_row_stride, q_dtype, E, e_row_stride, e_dtype, rstd,
                       dq, dq_row_stride, dq_dtype, dE, de_row_stride, de_dtype, rows, C, eps,
                       static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_layer_norm_fwd(const void* x, int x_dtype, const void* w, const void* b, int w_dtype,
                                  void* y, int y_dtype, float* mean, float* rstd, int64_t rows, int64_t C,
                                  double eps, void* stream) {
    clear_error();
    return layer_norm_fwd(x, x_dtype, nullptr, 0, nullptr, w, b, w_dtype, y, y_dtype, mean, rstd, rows, C, eps,
                          static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_add_layer_norm_fwd(const void* x, int x_dtype, const void* res, int res_dtype, void* xsum,
                                      const void* w, const void* b, int w_dtype, void* y, int y_dtype,
                                      float* mean, float* rstd, int64_t rows, int64_t C, double eps,
                                      void* stream) {
    clear_error();
    if (res == nullptr || xsum == nullptr)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "add layer norm: null res or xsum");
    return layer_norm_fwd(x, x_dtype, res, res_dtype, xsum, w, b, w_dtype, y, y_dtype, mean, rstd, rows, C,
                          eps, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT size_t esa_layer_norm_workspace_bytes(int64_t rows, int64_t C) {
    if (rows < 0 || C <= 0) return 0;
    return (size_t)layer_norm_partial_rows(rows > 0 ? rows : 1) * 2 * (size_t)C * sizeof(float);
}

static int ln_workspace_ok(void* workspace, size_t workspace_bytes, int64_t rows, int64_t C) {
    const size_t need = (size_t)layer_norm_partial_rows(rows > 0 ? rows : 1) * 2 * (size_t)(C > 0 ? C : 0) *
                        sizeof(float);
    if (workspace == nullptr || workspace_bytes < need)
        return set_error(ESA_ERR_WORKSPACE, "layer norm backward: workspace smaller than esa_layer_norm_workspace_bytes()");
    return ESA_OK;
}

ESA_EXPORT int esa_layer_norm_bwd(const void* dy, int dy_dtype, const void* x, int x_dtype, const void* w,
                                  int w_dtype, const float* mean, const float* rstd, void* dx, void* dw,
                                  void* db, void* workspace, size_t workspace_bytes, int64_t rows, int64_t C,
                                  void* stream) {
    clear_error();
    if (int rc = ln_workspace_ok(workspace, workspace_bytes, rows, C)) return rc;
    return layer_norm_bwd(dy, dy_dtype, nullptr, 0, x, x_dtype, w, w_dtype, mean, rstd, dx, nullptr, 0, dw, db,
                          static_cast<float*>(workspace), rows, C, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_add_layer_norm_bwd(const void* dy, int dy_dtype, const void* dsum, int dsum_dtype,
                                      const void* xsum, int x_dtype, const void* w, int w_dtype,
                                      const float* mean, const float* rstd, void* dx, void* dres,
                                      int res_dtype, void* dw, void* db, void* workspace,
                                      size_t workspace_bytes, int64_t rows, int64_t C, void* stream) {
    clear_error();
    if (int rc = ln_workspace_ok(workspace, workspace_bytes, rows, C)) return rc;
    return layer_norm_bwd(dy, dy_dtype, dsum, dsum_dtype, xsum, x_dtype, w, w_dtype, mean, rstd, dx, dres,
                          res_dtype, dw, db, static_cast<float*>(workspace), rows, C,
                          static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_wait_selftest(unsigned int* completed, unsigned int* waited_ms, void* stream) {
    clear_error();
    return wait_selftest(completed, waited_ms, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_device_status(int device, int clear, unsigned int* status) {
    clear_error();
    if (status == nullptr) return set_error(ESA_ERR_INVALID_ARGUMENT, "status pointer is null");
    return device_status(device, clear, status);
}

ESA_EXPORT size_t esa_scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int dtype, int compass) {
    const int es = dtype_size(dtype);
    if (es == 0 || nb < 0 || T < 0 || hd < 0 || compass <= 0) return 0;
    return scan_workspace_bytes(nb, T, hd, es, compass);
}

ESA_EXPORT size_t esa_layer_workspace_bytes(int64_t nb, int64_t T, int64_t C, int qgv_dtype, int e_dtype,
                                            int y_dtype) {
    return layer_workspace_bytes(nb, T, C, qgv_dtype, e_dtype, y_dtype);
}

ESA_EXPORT int esa_layer_fwd(const void* qgv, int64_t qgv_row_stride, int qgv_dtype, void* E, int e_dtype, void* y,
                             int y_dtype, void* rstd, int64_t nb, int64_t T, int64_t C, double gate_min,
                             double gate_max, double eps, const void* e0, void* e_last, void* workspace,
                             size_t workspace_bytes, void* stream) {
    clear_error();
    return layer_fwd(qgv, qgv_row_stride, qgv_dtype, E, e_dtype, y, y_dtype, rstd, nb, T, C, gate_min, gate_max, eps,
                     e0, e_last, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_layer_bwd(const void* dy, int dy_dtype, const void* qgv, int64_t qgv_row_stride, int qgv_dtype,
                             const void* E, int e_dtype, const void* rstd, void* dqgv, int64_t dqgv_row_stride,
                             int64_t nb, int64_t T, int64_t C, double gate_min, double gate_max, double eps,
                             const void* e0, void* de0, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    return layer_bwd(dy, dy_dtype, qgv, qgv_row_stride, qgv_dtype, E, e_dtype, rstd, dqgv, dqgv_row_stride, nb, T, C,
                     gate_min, gate_max, eps, e0, de0, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_scan_fwd(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd,
                 int dtype, int compass, const void* e0, void* e_last, void* workspace,
                 size_t workspace_bytes, void* stream) {
    clear_error();
    return scan_fwd(A, B, E, nb, T, hd, dtype, compass, e0, e_last, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}

ESA_EXPORT size_t esa_scan_host_staging_bytes(int64_t nb, int64_t T, int64_t hd, int dtype, int compass) {
    const int es = dtype_size(dtype);
    if (es == 0 || nb < 0 || T < 0 || hd < 0 || compass <= 0) return 0;
    return scan_host_staging_bytes(nb, T, hd, es, compass);
}

ESA_EXPORT int esa_scan_fwd_host(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd,
                                 int dtype, int compass, void* staging, size_t staging_bytes, void* stream) {
    clear_error();
    return scan_fwd_host(A, B, E, nb, T, hd, dtype, compass, staging, staging_bytes,
                         static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_scan_fwd_resume(const void* A, const void* B, void* E, int64_t nb, int64_t T,
                                   int64_t hd, int dtype, int compass, const void* e0, void* e_last,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    return scan_fwd(A, B, E, nb, T, hd, dtype, compass, e0, e_last, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream), true);
}

ESA_EXPORT int esa_scan_summary(const void* A, const void* B, int64_t nb, int64_t T, int64_t hd,
                                int dtype, const void* e0, void* e_last, void* prod, void* workspace,
                                size_t workspace_bytes, void* stream) {
    clear_error();
    return scan_summary(A, B, nb, T, hd, dtype, e0, e_last, prod, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_scan_prod(const void* A, void* prod, int64_t nb, int64_t T, int64_t hd, int dtype,
                             void* stream) {
    clear_error();
    return scan_prod(A, prod, nb, T, hd, dtype, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_scan_fixup(const void* A, const void* B, void* E, const void* carry, int64_t nb, int64_t T,
                              int64_t hd, int dtype, void* stream) {
    clear_error();
    return scan_fixup(A, B, E, carry, nb, T, hd, dtype, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_scan_rev(const void* A, const void* E, const void* dE, void* dA, void* dB, int64_t nb,
                 int64_t T, int64_t hd, int dtype, int compass, const void* e0, void* de0,
                 void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    return scan_rev(A, E, dE, dA, dB, nb, T, hd, dtype, compass, e0, de0, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_gated_scan_fwd(const void* gate_raw, const void* value_raw, int64_t raw_row_stride,
                       int raw_dtype, void* E, int e_dtype, int64_t nb, int64_t T, int64_t hd,
                       double gate_min, double gate_max, int round_ab, int compass, const void* e0,
                       void* e_last, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    return gated_scan_fwd(gate_raw, value_raw, raw_row_stride, raw_dtype, E, e_dtype, nb, T, hd,
                          gate_min, gate_max, round_ab, compass, e0, e_last, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_gated_scan_bwd(const void* gate_raw, const void* value_raw, int64_t raw_row_stride,
                       int raw_dtype, const void* E, const void* dE, int e_dtype,
                       void* d_gate_raw, void* d_value_raw, int64_t draw_row_stride,
                       int draw_dtype, int64_t nb, int64_t T, int64_t hd, double gate_min,
                       double gate_max, int round_ab, int compass, const void* e0, void* de0,
                       void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    return gated_scan_bwd(gate_raw, value_raw, raw_row_stride, raw_dtype, E, dE, e_dtype,
                          d_gate_raw, d_value_raw, draw_row_stride, draw_dtype, nb, T, hd,
                          gate_min, gate_max, round_ab, compass, e0, de0, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_lightning_step(const void* qgv, int64_t qgv_row_stride, int qgv_dtype, const void* state,
                       void* new_state, int state_dtype, void* z, int z_dtype, int64_t nb,
                       int64_t C, double gate_min, double gate_max, double eps, void* stream) {
    clear_error();
    return lightning_step(qgv, qgv_row_stride, qgv_dtype, state, new_state, state_dtype, z, z_dtype,
                          nb, C, gate_min, gate_max, eps, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT size_t esa_decode_block_scratch_bytes(int64_t nb, int64_t C, int dtype) {
    return decode_block_scratch_bytes(nb, C, dtype);
}

ESA_EXPORT int esa_decode_block(const void* x, const void* pending, void* x_out, void* pending_out,
                                const void* state, void* new_state, const void* ln1_w, const void* ln1_b,
                                const void* qgv_w, const void* qgv_b, const void* out_w, const void* out_b,
                                const void* ln2_w, const void* ln2_b, const void* fc_w, const void* fc_b,
                                const void* proj_w, const void* proj_b, int64_t nb, int64_t C, int dtype,
                                double gate_min, double gate_max, double eps, double ln_eps, void* scratch,
                                size_t scratch_bytes, void* stream) {
    clear_error();
    DecodeBlock p{};
    p.x = x;
    p.pending = pending;
    p.x_out = x_out;
    p.pending_out = pending_out;
    p.state = state;
    p.new_state = new_state;
    p.ln1_w = ln1_w;
    p.ln1_b = ln1_b;
    p.qgv_w = qgv_w;
    p.qgv_b = qgv_b;
    p.out_w = out_w;
    p.out_b = out_b;
    p.ln2_w = ln2_w;
    p.ln2_b = ln2_b;
    p.fc_w = fc_w;
    p.fc_b = fc_b;
    p.proj_w = proj_w;
    p.proj_b = proj_b;
    p.scratch = scratch;
    p.scratch_bytes = scratch_bytes;
    p.nb = nb;
    p.C = C;
    p.dtype = dtype;
    p.gate_min = gate_min;
    p.gate_max = gate_max;
    p.eps = eps;
    p.ln_eps = ln_eps;
    return decode_block(p, static_cast<cudaStream_t>(stream));
}

ESA_EXPORT int esa_decode_head(const void* x, const void* pending, const void* ln_w, const void* ln_b,
                               double ln_eps, const void* W, const void* bias, void* logits, int64_t nb, int64_t C,
                               int64_t V, int dtype, void* stream) {
    clear_error();
    return decode_head(x, pending, ln_w, ln_b, ln_eps, W, bias, logits, nb, C, V, dtype,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"
