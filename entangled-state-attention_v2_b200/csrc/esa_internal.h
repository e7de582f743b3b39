// esa_internal.h -- host-side declarations shared by the library's translation
// units, and the plain argument structs the scan kernels receive.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace esa {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
// Clears this thread's last error.
void clear_error();
// Kernel family of the last scan launch on this host thread (ESA_PATH_*).
void note_scan_path(int path);
int last_scan_path();
// Number of SMs of `device` (cached).
int device_sm_count(int device);
// Device address of the status word on `device` (cached; null on failure).
unsigned* status_ptr(int device);
int device_status(int device, int clear, unsigned* status);

inline int dtype_size(int dtype) {
    switch (dtype) {
        case 0: return 2;
        case 1: return 2;
        case 2: return 4;
        case 3: return 8;
        default: return 0;
    }
}

// FwdSummary: the forward recurrence over [0, T) reduced to its per-channel
// end state and product of A (no per-step outputs): the summary of a time
// slice, for composing slices held by different GPUs.
enum class Kind { FwdPlain, FwdGated, RevPlain, RevGated, FwdSummary };

// A row-strided view: element (row, c) at p + (row * rs + c) * elem_size,
// row = b * T + t.
struct View {
    const char* p;
    int64_t rs;
};
struct MutView {
    char* p;
    int64_t rs;
};

// Arguments common to every scan kernel (trivially copyable).
struct KArgs {
    View in[4];
    MutView out[2];
    int64_t nb, T, hd;
    const void* e0;    // acc [nb*hd] or null
    void* e_last;      // fwd: E_{T-1}; rev: gradient w.r.t. e0 (acc [nb*hd]) or null
    void* prod_out;    // summary passes: product of the step coefficients (acc [rows*hd])
    const void* cin;   // split passes: incoming state per (row, piece) (acc [nb*npiece*hd]) or null
    double gmin, span; // gate_min and gate_max - gate_min
    int round_ab;
    unsigned* status;  // device status word
};

// One scan call after argument checks: kind, element types, arguments.
struct ScanCall {
    Kind kind;
    int tin, te;  // dtype codes of staged logits / A (tin) and of E (te)
    KArgs a;
    int compass;
    void* ws;
    size_t ws_bytes;
    cudaStream_t stream;
    bool bulk_ok;  // every row 16-byte aligned (TMA-stageable)
    // time split: each batch row cut into npiece pieces of plen steps (a
    // multiple of 64), processed as independent rows of the strip scan
    int64_t npiece = 1, plen = 0;
    bool summ = false;  // summary pass: end state and coefficient product, no outputs
    // split scans: the workspace already holds this problem's piece summaries
    // (from a summary call on the same inputs): skip the summary pass
    bool resume = false;
};

// Channel-strip scan (no inter-CTA waits).  Sets *taken = false when the
// problem has too few channels to fill the GPU with strips.
int strip_scan_launch(const ScanCall& c, bool* taken);
// Single-pass chained scan of time pieces (esa_chain.cu): the plain forward
// scan of few channels over a long time axis.  Sets *taken = false when the
// shape is not one it serves or the workspace is smaller than
// chain_workspace_bytes.
int chain_scan_launch(const ScanCall& c, bool* taken);
size_t chain_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int es);
bool chain_applies_dims(int64_t nb, int64_t T, int64_t hd, int es);
// Time-chunked scan with decoupled lookback (any shape with aligned rows).
int lookback_scan_launch(const ScanCall& c);
// Sequential per-channel scan (any shape, any alignment).
int sequential_scan_launch(const ScanCall& c);
size_t lookback_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass);

int scan_fwd(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
             int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes, cudaStream_t s,
             bool resume = false);
int scan_rev(const void* A, const void* E, const void* dE, void* dA, void* dB, int64_t nb, int64_t T,
             int64_t hd, int dtype, int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
             cudaStream_t s);
int gated_scan_fwd(const void* g, const void* v, int64_t rrs, int raw_dtype, void* E, int e_dtype,
                   int64_t nb, int64_t T, int64_t hd, double gmin, double gmax, int round_ab,
                   int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes,
                   cudaStream_t s);
int gated_scan_bwd(const void* g, const void* v, int64_t rrs, int raw_dtype, const void* E,
                   const void* dE, int e_dtype, void* dg, void* dv, int64_t drs, int draw_dtype,
                   int64_t nb, int64_t T, int64_t hd, double gmin, double gmax, int round_ab,
                   int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
                   cudaStream_t s);
int scan_summary(const void* A, const void* B, int64_t nb, int64_t T, int64_t hd, int dtype,
                 const void* e0, void* e_last, void* prod, void* ws, size_t ws_bytes, cudaStream_t s);
int scan_prod(const void* A, void* prod, int64_t nb, int64_t T, int64_t hd, int dtype, cudaStream_t s);
int scan_fixup(const void* A, const void* B, void* E, const void* carry, int64_t nb, int64_t T, int64_t hd,
               int dtype, cudaStream_t s);
size_t scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass);
size_t scan_host_staging_bytes(int64_t nb, int64_t T, int64_t hd, int es, int compass);
int scan_fwd_host(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
                  int compass, void* staging, size_t staging_bytes, cudaStream_t s);
int wait_selftest(unsigned* completed, unsigned* waited_ms, cudaStream_t s);
int layer_norm_partial_rows(int64_t rows);
int layer_norm_fwd(const void* x, int xdt, const void* res, int rdt, void* xsum, const void* w,
                   const void* b, int wdt, void* y, int ydt, float* mean, float* rstd, int64_t rows, int64_t C,
                   double eps, cudaStream_t s);
int layer_norm_bwd(const void* dy, int dydt, const void* dsum, int dsdt, const void* x, int xdt,
                   const void* w, int wdt, const float* mean, const float* rstd, void* dx, void* dres, int rdt,
                   void* dw, void* db, float* partial, int64_t rows, int64_t C, cudaStream_t s);
int readout_fwd(const void* q, int64_t qrs, int qdt, const void* E, int64_t ers, int edt, void* y,
                int64_t yrs, int ydt, void* rstd, int64_t rows, int64_t C, double eps, cudaStream_t s);
int readout_bwd(const void* dy, int64_t dyrs, int dydt, const void* q, int64_t qrs, int qdt, const void* E,
                int64_t ers, int edt, const void* rstd, void* dq, int64_t dqrs, int dqdt, void* dE,
                int64_t ders, int dedt, int64_t rows, int64_t C, double eps, cudaStream_t s);
int cross_entropy_fwd(const void* logits, int64_t ld, int dtype, const int64_t* targets, int64_t ignore_index,
                      float* lse, float* loss, int64_t rows, int64_t V, cudaStream_t s);
int cross_entropy_bwd(const void* logits, int64_t ld, int dtype, const int64_t* targets, int64_t ignore_index,
                      const float* lse, const float* grad_rows, void* dlogits, int64_t dld, int64_t rows, int64_t V,
                      cudaStream_t s);
// ESA layer core (esa_layer.cu): the gated scan and the RMS readout kernels
// in turn (forward), the readout backward and the reverse gated scan.
size_t layer_workspace_bytes(int64_t nb, int64_t T, int64_t C, int qdt, int edt, int ydt);
int layer_fwd(const void* qgv, int64_t qrs, int qdt, void* E, int edt, void* y, int ydt, void* rstd, int64_t nb,
              int64_t T, int64_t C, double gmin, double gmax, double eps, const void* e0, void* e_last, void* ws,
              size_t ws_bytes, cudaStream_t s);
int layer_bwd(const void* dy, int dydt, const void* qgv, int64_t qrs, int qdt, const void* E, int edt,
              const void* rstd, void* dqgv, int64_t dqrs, int64_t nb, int64_t T, int64_t C, double gmin, double gmax,
              double eps, const void* e0, void* de0, void* ws, size_t ws_bytes, cudaStream_t s);
int lightning_step(const void* qgv, int64_t qrs, int qdt, const void* state, void* new_state,
                   int sdt, void* z, int zdt, int64_t nb, int64_t C, double gmin, double gmax,
                   double eps, cudaStream_t s);

// ESAModel block decode step for a few rows of 16-bit data (esa_decode.cu).
constexpr int kDecodeMaxRows = 4;
struct DecodeBlock {
    const void *x, *pending;            // [nb, C]; pending nullable (first block)
    void *x_out, *pending_out;          // [nb, C]
    const void* state;                  // [nb, C]
    void* new_state;                    // [nb, C], not aliasing state
    const void *ln1_w, *ln1_b, *qgv_w, *qgv_b, *out_w, *out_b;
    const void *ln2_w, *ln2_b, *fc_w, *fc_b, *proj_w, *proj_b;  // biases nullable
    void* scratch;
    size_t scratch_bytes;
    int64_t nb, C;
    int dtype;
    double gate_min, gate_max, eps, ln_eps;
};
size_t decode_block_scratch_bytes(int64_t nb, int64_t C, int dtype);
int decode_block(const DecodeBlock& p, cudaStream_t s);
int decode_head(const void* x, const void* pending, const void* ln_w, const void* ln_b, double ln_eps,
                const void* W, const void* bias, void* logits, int64_t nb, int64_t C, int64_t V, int dtype,
                cudaStream_t s);

}  // namespace esa
