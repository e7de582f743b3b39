/*
 * esa_oracle.c -- CPU fp64 restatement of the ESA recurrence.  TEST
 * INFRASTRUCTURE ONLY: the test-suite, the smoke check and the CPU baseline leg
 * of bench.py call it as the checker.  Nothing in the product links it.
 *
 * Every function runs in double precision, one channel at a time, in the
 * reference's sequential order, so its results are the exact-arithmetic answer
 * up to fp64 rounding.  Parity pin: tests/test_oracle.py checks each function
 * against fixtures produced by running the reference package itself
 * (tests/golden/make_golden.py).
 *
 * Layout: every [B, T, H, D] tensor is addressed as [nb][T][hd] with hd = H*D
 * contiguous, exactly the reference's contiguous layout.
 *
 * Build: oracle/Makefile (gcc, -ffp-contract=off so that a*s + b rounds twice,
 * as PyTorch's CPU kernels do).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#define IDX(b, t, c) (((int64_t)(b) * T + (t)) * hd + (c))

/* Forward recurrence E_t = A_t * E_{t-1} + B_t with E_{-1} = e0 (or 0).
 * Follows esa/backends/pulse.py:25-31 (pulse_scan). */
void esa_oracle_scan_fwd(const double *A, const double *B, double *E,
                         int64_t nb, int64_t T, int64_t hd, const double *e0)
{
    int64_t nch = nb * hd;
#pragma omp parallel for schedule(static)
    for (int64_t ch = 0; ch < nch; ++ch) {
        int64_t b = ch / hd, c = ch % hd;
        double s = e0 ? e0[ch] : 0.0;
        for (int64_t t = 0; t < T; ++t) {
            int64_t i = IDX(b, t, c);
            s = A[i] * s + B[i];
            E[i] = s;
        }
    }
}

/* Reverse-time recurrence for the gradient of the forward scan.
 *   G_t  = dE_t + A_{t+1} * G_{t+1}      (G_T = 0)
 *   dB_t = G_t,  dA_t = G_t * E_{t-1}   (E_{-1} = e0 or 0)
 *   de0  = A_0 * G_0                     (gradient w.r.t. the initial state)
 * This is the math of esa/backends/flare.py:66-78 (the only hand-written
 * backward in the reference) and equals autograd through pulse.py:28-31. */
void esa_oracle_scan_rev(const double *A, const double *E, const double *dE,
                         double *dA, double *dB, int64_t nb, int64_t T,
                         int64_t hd, const double *e0, double *de0)
{
    int64_t nch = nb * hd;
#pragma omp parallel for schedule(static)
    for (int64_t ch = 0; ch < nch; ++ch) {
        int64_t b = ch / hd, c = ch % hd;
        double future = 0.0;
        for (int64_t t = T - 1; t >= 0; --t) {
            int64_t i = IDX(b, t, c);
            double g = dE[i] + future;
            double eprev = t > 0 ? E[IDX(b, t - 1, c)] : (e0 ? e0[ch] : 0.0);
            dB[i] = g;
            dA[i] = g * eprev;
            future = g * A[i];
        }
        if (de0)
            de0[ch] = future;
    }
}

static double sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }

/* Gate prologue of the layer: A = gmin + (gmax - gmin) * sigmoid(g),
 * B = (1 - A) * tanh(v).  esa/backends/thunder.py:282-286 (ThunderESA.forward),
 * pulse.py:78-81, generation.py:439-445. */
void esa_oracle_gate(const double *g, const double *v, double *A, double *Bw,
                     int64_t n, double gmin, double gmax)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        double a = gmin + (gmax - gmin) * sigmoid(g[i]);
        A[i] = a;
        Bw[i] = (1.0 - a) * tanh(v[i]);
    }
}

/* Chain rule of the gate prologue, from (dA, dB) to (d gate_raw, d value_raw):
 *   s = sigmoid(g), A = gmin + (gmax-gmin) s, V = tanh(v), B = (1-A) V
 *   dg = (dA - dB * V) * (gmax - gmin) * s * (1 - s)
 *   dv = dB * (1 - A) * (1 - V^2)
 * The derivative of thunder.py:282-286, which the reference leaves to autograd. */
void esa_oracle_gate_bwd(const double *g, const double *v, const double *dA,
                         const double *dB, double *dg, double *dv, int64_t n,
                         double gmin, double gmax)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        double s = sigmoid(g[i]);
        double a = gmin + (gmax - gmin) * s;
        double V = tanh(v[i]);
        dg[i] = (dA[i] - dB[i] * V) * (gmax - gmin) * s * (1.0 - s);
        dv[i] = dB[i] * (1.0 - a) * (1.0 - V * V);
    }
}

/* One ESA-Lightning decode step for nb rows of C = H*D channels.
 * qgv is [nb][3C] (q | gate_raw | value_raw), state/new_state are [nb][C],
 * z (the input of out_proj) is [nb][C]:
 *   S' = A * S + B;   z = sigmoid(q) * S' * rsqrt(mean(S'^2) + eps)
 * esa/generation.py:443-458 (lightning_decode_step) and :270-293 (_readout). */
void esa_oracle_lightning_step(const double *qgv, const double *state,
                               double *new_state, double *z, int64_t nb,
                               int64_t C, double gmin, double gmax, double eps)
{
    for (int64_t b = 0; b < nb; ++b) {
        const double *q = qgv + b * 3 * C;
        const double *gr = q + C;
        const double *vr = q + 2 * C;
        double ss = 0.0;
        for (int64_t c = 0; c < C; ++c) {
            double a = gmin + (gmax - gmin) * sigmoid(gr[c]);
            double bw = (1.0 - a) * tanh(vr[c]);
            double s = a * state[b * C + c] + bw;
            new_state[b * C + c] = s;
            ss += s * s;
        }
        double r = 1.0 / sqrt(ss / (double)C + eps);
        for (int64_t c = 0; c < C; ++c)
            z[b * C + c] = sigmoid(q[c]) * new_state[b * C + c] * r;
    }
}

/* RMS readout over all C channels of each (b, t) row (thunder.py:304-311):
 * z = sigmoid(q) * E * rsqrt(mean(E^2) + eps).  rows = nb*T. */
void esa_oracle_readout(const double *q, const double *E, double *z,
                        int64_t rows, int64_t C, double eps)
{
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        double ss = 0.0;
        for (int64_t c = 0; c < C; ++c)
            ss += E[r * C + c] * E[r * C + c];
        double inv = 1.0 / sqrt(ss / (double)C + eps);
        for (int64_t c = 0; c < C; ++c)
            z[r * C + c] = sigmoid(q[r * C + c]) * E[r * C + c] * inv;
    }
}

/* Single-threaded fp32 forward scan, the scalar CPU port used as a timed
 * baseline (same recurrence, fp32 state, channels outer, time inner). */
void esa_oracle_scan_fwd_f32(const float *A, const float *B, float *E,
                             int64_t nb, int64_t T, int64_t hd)
{
    for (int64_t b = 0; b < nb; ++b) {
        for (int64_t c = 0; c < hd; ++c) {
            float s = 0.0f;
            for (int64_t t = 0; t < T; ++t) {
                int64_t i = IDX(b, t, c);
                s = A[i] * s + B[i];
                E[i] = s;
            }
        }
    }
}
