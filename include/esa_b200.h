/*
 * esa_b200.h -- C ABI of the B200 (sm_100a) ESA recurrence library
 * (libesa_b200.so).
 *
 * The reference (maxzameer/Entangled-State-Attention_v2 v2.1.1) is a pure
 * Python/PyTorch package with no FFI of its own; these entry points are the
 * functions its Python hot path would bind.  Each declaration cites the
 * reference interface it replaces.
 *
 * Conventions
 *   - All pointers are device pointers (cudaMalloc / PyTorch CUDA tensors),
 *     except where noted.  The library never allocates or frees memory, never
 *     synchronises the host and enqueues all work on `stream` (a cudaStream_t
 *     passed as void*; NULL = legacy default stream).
 *   - Tensors of shape [B, T, H, D] are passed as (nb = B, T, hd = H*D) and are
 *     contiguous with hd the fastest axis, the reference's layout
 *     (esa/backends/thunder.py:97-110).
 *   - Return value: ESA_OK (0) or a negative ESA_ERR_* code; esa_last_error()
 *     gives a message (thread-local).  Failures detected on the device (a wait
 *     that ran past its one-second budget) are OR-ed into a per-device status
 *     word read by esa_device_status().
 *   - "acc" type: double if any tensor of the call is f64, else float.  Initial
 *     and final states (e0, e_last, de0) use the acc type, shape [nb, hd].
 *   - gate_min, gate_max, eps are doubles; kernels use (acc)gate_min and
 *     (acc)(gate_max - gate_min), the values PyTorch uses for
 *     `gate_min + (gate_max - gate_min) * sigmoid(g)` with Python-float bounds.
 */
#ifndef ESA_B200_H
#define ESA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element type codes */
#define ESA_DTYPE_F16 0
#define ESA_DTYPE_BF16 1
#define ESA_DTYPE_F32 2
#define ESA_DTYPE_F64 3

/* return codes */
#define ESA_OK 0
#define ESA_ERR_INVALID_ARGUMENT (-1)
#define ESA_ERR_UNSUPPORTED_DTYPE (-2)
#define ESA_ERR_WORKSPACE (-3)
#define ESA_ERR_CUDA (-4)

/* device status bits */
#define ESA_STATUS_LOOKBACK_TIMEOUT 1u
#define ESA_STATUS_COPY_TIMEOUT 2u

#define ESA_ABI_VERSION 1

/* ESA readout of `rows` rows of C channels, fused:
 *   y = sigmoid(q) * E * rsqrt(mean_C(E^2) + eps)
 * in fp32 (fp64 if any operand is fp64), one rounding per output.  Every
 * operand is a row-strided view of its own dtype (row strides in elements:
 * e.g. 3*C for the q slice of a qgv [.., 3C] projection); rstd receives the
 * per-row rsqrt ([rows], acc type) for esa_readout_bwd.  Replaces the readout
 * of ThunderESA.forward (esa/backends/thunder.py:304-311) and `_readout`
 * (esa/generation.py:270-293) up to the out_proj. */
int esa_readout_fwd(const void *q, int64_t q_row_stride, int q_dtype, const void *E,
                    int64_t e_row_stride, int e_dtype, void *y, int64_t y_row_stride, int y_dtype,
                    void *rstd, int64_t rows, int64_t C, double eps, void *stream);

/* Gradient of esa_readout_fwd: from dy, q, E and the forward's rstd,
 *   dq = dy * n * s * (1 - s),  dE = r * (dy * s - n * mean_C(dy * s * n)),
 * with s = sigmoid(q), r = rstd, n = E * r.  dq and dE are row-strided
 * outputs of their own dtypes (dq can be the q slice of a qgv gradient).
 * Replaces the autograd of the readout (esa/backends/thunder.py:304-311). */
int esa_readout_bwd(const void *dy, int64_t dy_row_stride, int dy_dtype, const void *q,
                    int64_t q_row_stride, int q_dtype, const void *E, int64_t e_row_stride,
                    int e_dtype, const void *rstd, void *dq, int64_t dq_row_stride, int dq_dtype,
                    void *dE, int64_t de_row_stride, int de_dtype, int64_t rows, int64_t C,
                    double eps, void *stream);

/* LayerNorm of `rows` contiguous rows of C channels (C a multiple of 8, at
 * most 2048; 16-byte aligned rows):
 *   y = (x - mean) / sqrt(var + eps) * w + b     (biased variance, fp32 math)
 * x, w/b and y each of their own dtype; y is rounded once from the fp32
 * result (e.g. straight to the autocast dtype the consuming Linear would cast
 * an fp32 result to).  mean and rstd ([rows] fp32) are kept for the backward.
 * Replaces the blocks' F.layer_norm (esa/model.py of the reference) in the
 * ESAModel residual stream. */
int esa_layer_norm_fwd(const void *x, int x_dtype, const void *w, const void *b, int w_dtype,
                       void *y, int y_dtype, float *mean, float *rstd, int64_t rows, int64_t C,
                       double eps, void *stream);

/* Scratch (bytes) of esa_layer_norm_bwd: per-CTA partial column sums. */
size_t esa_layer_norm_workspace_bytes(int64_t rows, int64_t C);

/* Gradient of esa_layer_norm_fwd: dx (x's dtype), dw and db (w's dtype) from
 * dy (own dtype), x, w and the forward's mean/rstd.  dw and db are reduced in a
 * fixed order (deterministic). */
int esa_layer_norm_bwd(const void *dy, int dy_dtype, const void *x, int x_dtype, const void *w,
                       int w_dtype, const float *mean, const float *rstd, void *dx, void *dw, void *db,
                       void *workspace, size_t workspace_bytes, int64_t rows, int64_t C, void *stream);

/* esa_layer_norm_fwd fused with the residual add before it:
 *   xsum = x + res   (written in x's dtype, rounded as a separate add is)
 *   y    = LayerNorm(xsum)
 * res has its own dtype (e.g. the fp16 output of a Linear under autocast added
 * to an fp32 residual stream).  Replaces `x = x + branch(...)` followed by
 * `ln(x)` in the ESAModel blocks (esa/model.py of the reference). */
int esa_add_layer_norm_fwd(const void *x, int x_dtype, const void *res, int res_dtype, void *xsum,
                           const void *w, const void *b, int w_dtype, void *y, int y_dtype, float *mean,
                           float *rstd, int64_t rows, int64_t C, double eps, void *stream);

/* Gradient of esa_add_layer_norm_fwd: dx = LayerNorm backward at xsum (+ dsum,
 * the gradient of xsum, when not NULL) in x's dtype; dres (nullable) the same
 * values in res's dtype; dw, db as esa_layer_norm_bwd. */
int esa_add_layer_norm_bwd(const void *dy, int dy_dtype, const void *dsum, int dsum_dtype,
                           const void *xsum, int x_dtype, const void *w, int w_dtype, const float *mean,
                           const float *rstd, void *dx, void *dres, int res_dtype, void *dw, void *db,
                           void *workspace, size_t workspace_bytes, int64_t rows, int64_t C, void *stream);

/* Diagnostic: runs the kernels' bounded mbarrier wait on a barrier that never
 * completes, on `stream`, and synchronises it.  The wait gives up after its
 * one-second budget: *completed = 0, *waited_ms = the time waited, and
 * ESA_STATUS_COPY_TIMEOUT is set in the device status word (clear it with
 * esa_device_status).  Lets a test check the timeout path without a fault or
 * a hang.  No reference counterpart. */
int esa_wait_selftest(unsigned int *completed, unsigned int *waited_ms, void *stream);

/* Cross-entropy of the LM head (the ESAModel training loss), forward.
 * Replaces `F.cross_entropy(logits.reshape(-1, V), targets, ignore_index=-1)`
 * of the reference's esa/model.py (ESAModel.forward) up to its mean: for each
 * row i of logits [rows, V] (row stride `row_stride` elements; f16, bf16 or
 * f32), lse[i] = log sum_j exp(logits[i, j]) and loss[i] = lse[i] -
 * logits[i, targets[i]] (fp32; 0 where targets[i] == ignore_index, NaN where a
 * target is out of [0, V)).  The caller averages loss over the rows that are
 * not ignored.  Reads the logits once; lse is kept for the backward. */
int esa_cross_entropy_fwd(const void *logits, int64_t row_stride, int dtype, const int64_t *targets,
                          int64_t ignore_index, float *lse, float *loss, int64_t rows, int64_t V,
                          void *stream);

/* Gradient of esa_cross_entropy_fwd: dlogits[i, j] = grad_rows[i] *
 * (exp(logits[i, j] - lse[i]) - [j == targets[i]]), zero on ignored rows,
 * written in the logits' dtype (row stride `dlogits_row_stride`).  grad_rows:
 * fp32 [rows], the gradient of the loss w.r.t. each row's loss[i] (for a mean
 * over n rows: the upstream gradient / n).  A row whose target is outside
 * [0, V) and not ignore_index gets NaN gradients (its loss is NaN). */
int esa_cross_entropy_bwd(const void *logits, int64_t row_stride, int dtype, const int64_t *targets,
                          int64_t ignore_index, const float *lse, const float *grad_rows, void *dlogits,
                          int64_t dlogits_row_stride, int64_t rows, int64_t V, void *stream);

/* Kernel family of the last scan launch on this host thread (diagnostics and
 * tests): ESA_PATH_NONE before any, ESA_PATH_SEQUENTIAL (one thread per
 * channel, any alignment), ESA_PATH_LOOKBACK (time chunks, decoupled
 * look-back), ESA_PATH_STRIP (channel strips, tile-parallel steps),
 * ESA_PATH_LANE (channel strips, one lane per channel vector walking the
 * steps in order), ESA_PATH_CHAIN (time pieces chained by a single-pass
 * look-back, each piece read from HBM once and re-read from L2).  A split
 * scan reports its output pass.  No reference counterpart. */
#define ESA_PATH_NONE 0
#define ESA_PATH_SEQUENTIAL 1
#define ESA_PATH_LOOKBACK 2
#define ESA_PATH_STRIP 3
#define ESA_PATH_LANE 4
#define ESA_PATH_CHAIN 5
int esa_scan_last_path(void);

/* Version of this ABI (ESA_ABI_VERSION). */
int esa_abi_version(void);

/* Message for the last failing call on this host thread ("" if none). */
const char *esa_last_error(void);

/* Reads the device status word of `device` into *status (host pointer);
 * clears it when `clear` is non-zero.  Synchronises that device.
 * Replaces nothing in the reference (it has no device code); it is how the
 * bounded waits of the scans report failure. */
int esa_device_status(int device, int clear, unsigned int *status);

/* Workspace bytes a scan call needs for this problem (lookback descriptors and
 * flags).  0 is never returned for a valid problem.  `compass` as in
 * esa_scan_fwd. */
size_t esa_scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int dtype, int compass);

/* Forward recurrence E_t = A_t * E_{t-1} + B_t, E_{-1} = e0 (NULL: zero).
 * A, B, E: [nb, T, hd] of `dtype`; accumulation in the acc type.
 * e_last (nullable): receives E_{T-1} in the acc type.
 * compass: the reference's Thunder chunk size (any positive int); here it
 * selects the time extent of one CTA tile (16, 32 or 64 steps, nearest) and
 * does not change results beyond fp32 summation order.
 * Replaces thunder_scan(A, B_write, compass) -- esa/backends/thunder.py:70-159
 * (and pulse_scan, esa/backends/pulse.py:12-31). */
int esa_scan_fwd(const void *A, const void *B, void *E, int64_t nb, int64_t T, int64_t hd,
                 int dtype, int compass, const void *e0, void *e_last, void *workspace,
                 size_t workspace_bytes, void *stream);

/* Scratch size of esa_scan_fwd_noalloc (bytes). */
#define ESA_NOALLOC_SCRATCH_BYTES (16u << 20)

/* esa_scan_fwd for callers that cannot allocate device memory -- e.g. a C
 * host program or a foreign-language binding that receives its input and
 * output buffers from elsewhere, or code whose device memory plan is fixed
 * before it runs.  Same arguments and results as esa_scan_fwd, without the
 * workspace: the time-parallel scan kernel takes its scratch from a fixed
 * array of ESA_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until the process exits.  Problems whose scratch
 * would exceed that size are rejected with ESA_ERR_WORKSPACE and a message.
 * The first call on each device looks the array's address up
 * (cudaGetSymbolAddress); make it before any stream capture.  All calls share
 * the array, so calls that overlap on the GPU (e.g. on two streams at once)
 * race.  No counterpart in the reference: it has no native code and no
 * allocator-free interface. */
int esa_scan_fwd_noalloc(const void *A, const void *B, void *E, int64_t nb, int64_t T, int64_t hd,
                         int dtype, int compass, const void *e0, void *e_last, void *stream);

/* Staging size (bytes) of esa_scan_fwd_host for this problem; 0 for invalid
 * arguments.  Bounded (about 300 MB) whatever the problem size. */
size_t esa_scan_host_staging_bytes(int64_t nb, int64_t T, int64_t hd, int dtype, int compass);

/* esa_scan_fwd on HOST buffers: A, B and E are host pointers ([nb, T, hd] of
 * `dtype`, page-locked for the copies to overlap; pageable memory works but
 * serialises), `staging` a 256-byte aligned device buffer of at least
 * esa_scan_host_staging_bytes().  The tensor moves through the device in
 * chunks of about 32 MB per array (whole rows, or time pieces of one row
 * chained through their end state): the host-to-device copy of one chunk, the
 * scan of the previous one (on `stream`) and the device-to-host copy of the
 * one before run concurrently on the two copy engines and the SMs.  Ordered
 * after the work already on `stream`; work queued on `stream` afterwards (an
 * event record, cudaStreamSynchronize) sees E complete.  The library's own two
 * copy streams are created on the first call per device.  Replaces
 * thunder_scan on CPU tensors (esa/backends/thunder.py:70-159), whose output
 * is a CPU tensor. */
int esa_scan_fwd_host(const void *A, const void *B, void *E, int64_t nb, int64_t T, int64_t hd,
                      int dtype, int compass, void *staging, size_t staging_bytes, void *stream);

/* Summary of a time slice: the per-channel end state E_{T-1} of the forward
 * recurrence (from e0, NULL: zero) and the product of A over [0, T), both in
 * the acc type, [nb, hd]; no per-step outputs (reads A and B once).  The
 * workspace (esa_scan_workspace_bytes, may be NULL) lets few-channel, long
 * slices split their time axis across the GPU.  Two
 * consecutive slices compose as E_end = prod2 * E_end1 + E_end2 (from zero),
 * which is how GPUs holding consecutive time slices of one sequence combine
 * their carries.  Replaces nothing in the reference (it has no multi-device
 * path); part of the sequence-parallel scan built on thunder_scan
 * (esa/backends/thunder.py:70-159). */
int esa_scan_summary(const void *A, const void *B, int64_t nb, int64_t T, int64_t hd, int dtype,
                     const void *e0, void *e_last, void *prod, void *workspace,
                     size_t workspace_bytes, void *stream);

/* Product of A over the time axis: prod[b*hd + c] = A[b,0,c] * ... *
 * A[b,T-1,c] in the acc type, [nb, hd].  Reads A from t = 0 and stops once
 * the running product is exactly zero for every channel of a block (gates
 * below one reach zero after a few thousand steps; A = 1 reads all of A).
 * No workspace.  With the end state of esa_scan_fwd from a zero state
 * (e_last), this is a time slice's summary for esa_scan_summary's
 * composition rule.  Replaces nothing in the reference (it has no
 * multi-device path); part of the single-pass sequence-parallel scan. */
int esa_scan_prod(const void *A, void *prod, int64_t nb, int64_t T, int64_t hd, int dtype,
                  void *stream);

/* Head of a time slice that esa_scan_fwd scanned from a zero state, rescanned
 * once its true incoming state `carry` (acc type, [nb, hd]) is known:
 *   E[b,t,c] = A[b,t,c] * x_{t-1} + B[b,t,c],  x_{-1} = carry[b*hd + c]
 * (fp32 / fp64 state, each output rounded once to `dtype`), for t from 0
 * until the product A[b,0,c] * ... * A[b,t,c] is exactly zero for every
 * channel of a block; from there on the outputs of the scan from zero equal
 * those from `carry` (to the rounding of the state) and are left as they
 * are.  Replaces nothing in the reference (it has no multi-device path);
 * part of the single-pass sequence-parallel scan (esa/parallel.py). */
int esa_scan_fixup(const void *A, const void *B, void *E, const void *carry, int64_t nb, int64_t T,
                   int64_t hd, int dtype, void *stream);

/* esa_scan_fwd of a slice whose summary esa_scan_summary has just computed,
 * with the same A, B, shape, dtype and workspace (and no other call using the
 * workspace in between).  Few-channel, long slices are scanned in time pieces
 * whose summaries the summary call left in the workspace; this call reuses
 * them, so the pair reads A and B twice in all (summary + scan) instead of
 * three times.  Other problems are scanned in full, as by esa_scan_fwd.  The
 * results are those of esa_scan_fwd on the same arguments.  No counterpart in
 * the reference: the second half of the sequence-parallel scan. */
int esa_scan_fwd_resume(const void *A, const void *B, void *E, int64_t nb, int64_t T, int64_t hd,
                        int dtype, int compass, const void *e0, void *e_last, void *workspace,
                        size_t workspace_bytes, void *stream);

/* Reverse-time scan: the gradient of esa_scan_fwd.
 *   G_t = dE_t + A_{t+1} G_{t+1};  dB_t = G_t;  dA_t = G_t * E_{t-1}
 * with E_{-1} = e0 (NULL: zero); de0 (nullable) receives A_0 * G_0, the
 * gradient w.r.t. e0, in the acc type.  All tensors [nb, T, hd] of `dtype`.
 * Replaces the autograd backward of thunder_scan (esa/backends/thunder.py:
 * 70-159 has none of its own); math of esa/backends/flare.py:49-78. */
int esa_scan_rev(const void *A, const void *E, const void *dE, void *dA, void *dB, int64_t nb,
                 int64_t T, int64_t hd, int dtype, int compass, const void *e0, void *de0,
                 void *workspace, size_t workspace_bytes, void *stream);

/* Forward scan with the gate prologue fused in.  gate_raw / value_raw are
 * row-strided views ([nb, T] rows of hd elements, `raw_row_stride` elements
 * apart -- e.g. 3*C for the gate and value slices of a qgv [B,T,3C] tensor)
 * of `raw_dtype`.  Per element:
 *   A = gmin + (gmax - gmin) * sigmoid(gate_raw),  B = (1 - A) * tanh(value_raw)
 * both rounded to `e_dtype` first when round_ab != 0 (the reference's
 * A.to(scan_dtype)), then E_t = A_t E_{t-1} + B_t written as `e_dtype`.
 * Replaces esa/backends/thunder.py:282-302 (ThunderESA.forward: gate, cast,
 * thunder_scan) and generation.py:439-445 + :476-487 (prefill). */
int esa_gated_scan_fwd(const void *gate_raw, const void *value_raw, int64_t raw_row_stride,
                       int raw_dtype, void *E, int e_dtype, int64_t nb, int64_t T, int64_t hd,
                       double gate_min, double gate_max, int round_ab, int compass, const void *e0,
                       void *e_last, void *workspace, size_t workspace_bytes, void *stream);

/* Backward of esa_gated_scan_fwd, fused: reverse scan plus the gate chain rule
 *   dg = (dA - dB * tanh v) * (gmax - gmin) * s (1 - s),  s = sigmoid(g)
 *   dv = dB * (1 - A) * (1 - tanh^2 v)
 * writing d_gate_raw / d_value_raw as row-strided views (`draw_row_stride`,
 * `draw_dtype`, e.g. slices of the qgv gradient).  E and dE: [nb, T, hd] of
 * e_dtype.  A is recomputed from gate_raw exactly as the forward did.
 * Replaces the autograd of thunder.py:282-302. */
int esa_gated_scan_bwd(const void *gate_raw, const void *value_raw, int64_t raw_row_stride,
                       int raw_dtype, const void *E, const void *dE, int e_dtype,
                       void *d_gate_raw, void *d_value_raw, int64_t draw_row_stride,
                       int draw_dtype, int64_t nb, int64_t T, int64_t hd, double gate_min,
                       double gate_max, int round_ab, int compass, const void *e0, void *de0,
                       void *workspace, size_t workspace_bytes, void *stream);

/* Workspace (bytes) of esa_layer_fwd / esa_layer_bwd for [nb, T, C] with
 * these dtypes: the gated scan's workspace plus the dE buffer between the
 * readout backward and the reverse scan.  0 for invalid arguments.  No
 * counterpart in the reference (it has no native code). */
size_t esa_layer_workspace_bytes(int64_t nb, int64_t T, int64_t C, int qgv_dtype, int e_dtype,
                                 int y_dtype);

/* The ESA layer core forward: from the qgv projection [nb, T, 3C]
 * (q | gate_raw | value_raw; rows `qgv_row_stride` elements apart, of
 * qgv_dtype) it computes
 *   A = gmin + (gmax - gmin) sigmoid(gate_raw),  B = (1 - A) tanh(value_raw)
 *   (both rounded to e_dtype, the reference's A.to(scan_dtype)),
 *   E_t = A_t E_{t-1} + B_t               (E_{-1} = e0, NULL: zero)
 *   y = sigmoid(q) * E * rsqrt(mean_C(E^2) + eps)
 * writing E ([nb, T, C] of e_dtype, kept for the backward), y ([nb, T, C] of
 * y_dtype), rstd ([nb*T], acc type: the per-row rsqrt) and, if not NULL,
 * e_last = E_{T-1} (acc [nb, C]).  Two launches on `stream`: the gated scan
 * (gates fused into the scan's loads) and the RMS readout (sigmoid(q) gate
 * fused).  Replaces ThunderESA.forward from the qgv
 * projection to the out_proj input (esa/backends/thunder.py:275-311: split,
 * gates, cast, thunder_scan, RMS readout, sigmoid(q) gate). */
int esa_layer_fwd(const void *qgv, int64_t qgv_row_stride, int qgv_dtype, void *E, int e_dtype,
                  void *y, int y_dtype, void *rstd, int64_t nb, int64_t T, int64_t C,
                  double gate_min, double gate_max, double eps, const void *e0, void *e_last,
                  void *workspace, size_t workspace_bytes, void *stream);

/* Backward of esa_layer_fwd: from dy ([nb, T, C] of dy_dtype), qgv,
 * E and rstd it writes d qgv ([nb, T, 3C] of qgv_dtype, rows
 * `dqgv_row_stride` apart):
 *   dq = dy n s (1 - s),  dE = r (dy s - n mean_C(dy s n))   (s = sigmoid(q),
 *   n = E r), the reverse scan G_t = dE_t + A_{t+1} G_{t+1}, and
 *   d gate_raw = (G E_{t-1} - G tanh v) (gmax - gmin) s_g (1 - s_g),
 *   d value_raw = G (1 - A)(1 - tanh^2 v),
 * with E_{-1} = e0 (NULL: zero) and de0 (nullable) = A_0 G_0, the gradient
 * w.r.t. e0.  Two launches: the readout backward (writes dq and dE into the
 * workspace) and the gated reverse scan (gate chain rule fused).  Replaces
 * the autograd of
 * esa/backends/thunder.py:275-311. */
int esa_layer_bwd(const void *dy, int dy_dtype, const void *qgv, int64_t qgv_row_stride,
                  int qgv_dtype, const void *E, int e_dtype, const void *rstd, void *dqgv,
                  int64_t dqgv_row_stride, int64_t nb, int64_t T, int64_t C, double gate_min,
                  double gate_max, double eps, const void *e0, void *de0, void *workspace,
                  size_t workspace_bytes, void *stream);

/* Scratch (bytes) of esa_decode_block for nb rows of C channels: 18 nb C
 * (the block's intermediate activations).  0 for invalid arguments.  No
 * counterpart in the reference (it has no native code). */
size_t esa_decode_block_scratch_bytes(int64_t nb, int64_t C, int dtype);

/* One ESAModel block's decode step for nb = 1..4 rows of 16-bit data (dtype
 * fp16 or bf16 for every tensor; C a multiple of 256), in four launches:
 *   s1 = x + pending (pending NULL: s1 = x),  h1 = LN1(s1),
 *   qgv = qgv_w h1 + qgv_b,  the Lightning step state -> new_state and its
 *   readout z (as esa_lightning_step),  y = out_w z + out_b,
 *   x_out = s1 + y,  h2 = LN2(x_out),  a = GELU(fc_w h2 + fc_b),
 *   pending_out = proj_w a + proj_b.
 * Activations are [nb, C] (qgv [nb, 3C], a [nb, 4C] in the scratch),
 * weights are PyTorch Linear layouts ([out, in], row-major), every bias and
 * LayerNorm bias may be NULL; the four weight matrices must start on a
 * 16-byte boundary.  Each result is rounded to the 16-bit dtype
 * where the PyTorch path rounds it (fp32 accumulation).  new_state must not
 * alias state; x_out may alias x and pending_out pending.  The caller adds
 * the last block's pending_out (esa_decode_head does).  Replaces one block of
 * ESAModel.lightning_step (esa/model.py:717-757: ln_1, ESA.decode_step =
 * esa/generation.py:410-469, residual add, ln_2, MLP, residual add). */
int esa_decode_block(const void *x, const void *pending, void *x_out, void *pending_out,
                     const void *state, void *new_state, const void *ln1_w, const void *ln1_b,
                     const void *qgv_w, const void *qgv_b, const void *out_w, const void *out_b,
                     const void *ln2_w, const void *ln2_b, const void *fc_w, const void *fc_b,
                     const void *proj_w, const void *proj_b, int64_t nb, int64_t C, int dtype,
                     double gate_min, double gate_max, double eps, double ln_eps, void *scratch,
                     size_t scratch_bytes, void *stream);

/* The decode step's head: logits [nb, V] = W LN_f(x + pending) + bias
 * (pending and bias nullable; W [V, C], the tied embedding matrix), same
 * dtypes and limits as esa_decode_block.  Replaces ESAModel.lightning_step's
 * ln_f and lm_head (esa/model.py:717-757). */
int esa_decode_head(const void *x, const void *pending, const void *ln_w, const void *ln_b, double ln_eps,
                    const void *W, const void *bias, void *logits, int64_t nb, int64_t C, int64_t V,
                    int dtype, void *stream);

/* One ESA-Lightning decode step for nb rows, fused: gate nonlinearity, state
 * update and the RMS readout over all C = H*D channels.
 *   qgv: [nb, 3C] rows `qgv_row_stride` elements apart (q | gate | value)
 *   state -> new_state: [nb, C] of state_dtype (may alias)
 *   z: [nb, C] of z_dtype, z = sigmoid(q) * S' * rsqrt(mean(S'^2) + eps),
 *      the input of out_proj.
 * Replaces esa/generation.py:443-458 (lightning_decode_step: gates, S' =
 * A S + B, _readout up to out_proj; _readout is generation.py:270-293). */
int esa_lightning_step(const void *qgv, int64_t qgv_row_stride, int qgv_dtype,
                       const void *state, void *new_state, int state_dtype, void *z,
                       int z_dtype, int64_t nb, int64_t C, double gate_min, double gate_max,
                       double eps, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ESA_B200_H */
