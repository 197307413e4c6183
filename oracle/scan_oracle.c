/*
 * scan_oracle.c -- CPU oracle for the N-state selective scan and the first-order
 * linear recurrence.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg may load it.
 * The product path (mamba_windows_cuda + libmwc_b200.so) never calls it, and the
 * product fails loudly instead of falling back to it.
 *
 * Everything here is double precision and restates the reference's algorithm:
 *
 *   mamba_windows_cuda/mamba_cuda.py:875-946  selective_scan_ref: h_t = exp(dt_t*A) h_{t-1}
 *       + dt_t*u_t*B_t, y_t = <C_t, h_t> + D*u_t, h_{-1} = h_prev or 0, h_last = h_{L-1}.
 *       The einsum at :910 is read with the time axis last ('bdl,dn->bdnl'); that is the
 *       only reading under which the loop at :920-922 is the recurrence the CUDA kernels
 *       at :93-174 / :611-667 compute.
 *   mamba_windows_cuda/mamba_cuda.py:65-70    safe_exp: the CUDA kernels clamp the exponent
 *       to [-88, 88]; `clamp` != 0 reproduces that. As in the reference's CUDA backward
 *       (:724-731), the gradient terms use the clamped factor a with the unclamped
 *       formulas (d a / d delta taken as A a everywhere).
 *   mamba_windows_cuda/mamba_cuda.py:669-745  the gradients of that recurrence (bwd_direct),
 *       extended with dh_last in and dh_prev out, which the reference's stateful path
 *       (:1044-1096) promises but computes incorrectly.
 *   mamba_windows_cuda/pscan.py:153-171       parallel_scan_ref: H_0 = X_0,
 *       H_t = A_t H_{t-1} + X_t along dim 2 of (B, D, L, N); the gradient is the one
 *       PScan.backward (:98-136) intends: gX_t = g_t + A_{t+1} gX_{t+1}, gA_t = gX_t H_{t-1}.
 *
 * Parity of this restatement is pinned by tests/test_oracle.py against
 * the fixtures under tests/golden, which tests/golden/make_golden.py produced by running the
 * reference's own Python functions (selective_scan_ref + torch autograd,
 * parallel_scan_ref, and the closed form in tests/test_selective_scan.py:8-36).
 *
 * Layouts (all contiguous, row-major):
 *   u, delta, out, du, ddelta : (B, L, D)      A, dA : (D, N)
 *   Bm, Cm, dB, dC            : (B, L, N)      Dv, dD : (D)
 *   h_prev, h_last, dh_last, dh_prev : (B, D, N)
 *   linear scan a, x, h, g, ga, gx   : (R, L, N) with R = B*D rows
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

static inline double clamp_arg(double x, int clamp, int* inside) {
    if (!clamp) { *inside = 1; return x; }
    if (x < -88.0) { *inside = 0; return -88.0; }
    if (x > 88.0) { *inside = 0; return 88.0; }
    *inside = 1;
    return x;
}

ORC_EXPORT int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

ORC_EXPORT void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Forward selective scan (mamba_cuda.py:875-946 / :93-174). */
ORC_EXPORT void orc_ss_fwd(const double* u, const double* delta, const double* A,
                           const double* Bm, const double* Cm, const double* Dv,
                           const double* h_prev, double* out, double* h_last,
                           int64_t B, int64_t L, int64_t D, int64_t N, int clamp) {
    int64_t pairs = B * D;
#pragma omp parallel
    {
        double* h = (double*)malloc(sizeof(double) * (size_t)N);
#pragma omp for schedule(static)
        for (int64_t p = 0; p < pairs; ++p) {
            int64_t b = p / D, d = p % D;
            for (int64_t n = 0; n < N; ++n)
                h[n] = h_prev ? h_prev[(b * D + d) * N + n] : 0.0;
            for (int64_t t = 0; t < L; ++t) {
                int64_t i = (b * L + t) * D + d;
                double dt = delta[i], uu = u[i];
                const double* Bt = Bm + (b * L + t) * N;
                const double* Ct = Cm + (b * L + t) * N;
                double y = 0.0;
                for (int64_t n = 0; n < N; ++n) {
                    int inside;
                    double a = exp(clamp_arg(dt * A[d * N + n], clamp, &inside));
                    h[n] = a * h[n] + dt * uu * Bt[n];
                    y += Ct[n] * h[n];
                }
                out[i] = y + Dv[d] * uu;
            }
            if (h_last)
                for (int64_t n = 0; n < N; ++n) h_last[(b * D + d) * N + n] = h[n];
        }
        free(h);
    }
}

/*
 * Backward of orc_ss_fwd for loss = sum(out * dout) + sum(h_last * dh_last).
 * Per (b, d) channel: recompute every state, then run the adjoint recurrence
 *   g_t = dout_t * C_t + a_{t+1} * g_{t+1}     (g_{L-1} also receives dh_last)
 *   dC_t += dout_t h_t ;  dB_t += g_t dt_t u_t ;  du_t = dout_t D + dt_t <g_t, B_t>
 *   ddelta_t = <g_t, A a_t h_{t-1}> + u_t <g_t, B_t> ;  dA += g_t dt_t a_t h_{t-1}
 *   dD += dout_t u_t ;  dh_prev = a_0 g_0
 * (the per-step terms of mamba_cuda.py:703-742, with h_{-1} = h_prev).
 * dA/dD reduce over (b, t) and dB/dC over d; the sums are taken in a fixed order
 * (per-thread partials combined in thread order) so results are reproducible.
 */
ORC_EXPORT void orc_ss_bwd(const double* u, const double* delta, const double* A,
                           const double* Bm, const double* Cm, const double* Dv,
                           const double* h_prev, const double* dout, const double* dh_last,
                           double* du, double* ddelta, double* dA, double* dB, double* dC,
                           double* dD, double* dh_prev,
                           int64_t B, int64_t L, int64_t D, int64_t N, int clamp) {
    int nth = orc_num_threads();
    size_t bln = (size_t)(B * L * N);
    double* pB = (double*)calloc((size_t)nth * bln, sizeof(double));
    double* pC = (double*)calloc((size_t)nth * bln, sizeof(double));
    memset(dA, 0, sizeof(double) * (size_t)(D * N));
    memset(dD, 0, sizeof(double) * (size_t)D);
#pragma omp parallel num_threads(nth)
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        double* myB = pB + (size_t)tid * bln;
        double* myC = pC + (size_t)tid * bln;
        double* hs = (double*)malloc(sizeof(double) * (size_t)((L + 1) * N));
        double* q = (double*)malloc(sizeof(double) * (size_t)N);
        /* d outer so dA[d,:] and dD[d] are owned by exactly one thread */
#pragma omp for schedule(static)
        for (int64_t d = 0; d < D; ++d) {
            for (int64_t b = 0; b < B; ++b) {
                /* hs[0] = h_{-1}; hs[t+1] = h_t */
                for (int64_t n = 0; n < N; ++n)
                    hs[n] = h_prev ? h_prev[(b * D + d) * N + n] : 0.0;
                for (int64_t t = 0; t < L; ++t) {
                    int64_t i = (b * L + t) * D + d;
                    double dt = delta[i], uu = u[i];
                    const double* Bt = Bm + (b * L + t) * N;
                    for (int64_t n = 0; n < N; ++n) {
                        int inside;
                        double a = exp(clamp_arg(dt * A[d * N + n], clamp, &inside));
                        hs[(t + 1) * N + n] = a * hs[t * N + n] + dt * uu * Bt[n];
                    }
                }
                for (int64_t n = 0; n < N; ++n)
                    q[n] = dh_last ? dh_last[(b * D + d) * N + n] : 0.0;
                for (int64_t t = L - 1; t >= 0; --t) {
                    int64_t i = (b * L + t) * D + d;
                    double dt = delta[i], uu = u[i], gy = dout[i];
                    const double* Bt = Bm + (b * L + t) * N;
                    const double* Ct = Cm + (b * L + t) * N;
                    double* dBt = myB + (b * L + t) * N;
                    double* dCt = myC + (b * L + t) * N;
                    double s_gB = 0.0, s_dA = 0.0;
                    for (int64_t n = 0; n < N; ++n) {
                        int inside;
                        double arg = clamp_arg(dt * A[d * N + n], clamp, &inside);
                        double a = exp(arg);
                        double gn = gy * Ct[n] + q[n];
                        double hprev = hs[t * N + n];
                        double ah = a * hprev;
                        (void)inside;
                        dCt[n] += gy * hs[(t + 1) * N + n];
                        dBt[n] += gn * dt * uu;
                        s_gB += gn * Bt[n];
                        s_dA += gn * A[d * N + n] * ah;
                        dA[d * N + n] += gn * dt * ah;
                        q[n] = a * gn;
                    }
                    du[i] = gy * Dv[d] + dt * s_gB;
                    ddelta[i] = s_dA + uu * s_gB;
                    dD[d] += gy * uu;
                }
                if (dh_prev)
                    for (int64_t n = 0; n < N; ++n) dh_prev[(b * D + d) * N + n] = q[n];
            }
        }
        free(hs);
        free(q);
    }
    for (size_t k = 0; k < bln; ++k) {
        double sb = 0.0, sc = 0.0;
        for (int t = 0; t < nth; ++t) {
            sb += pB[(size_t)t * bln + k];
            sc += pC[(size_t)t * bln + k];
        }
        dB[k] = sb;
        dC[k] = sc;
    }
    free(pB);
    free(pC);
}

/* First-order linear recurrence along L (pscan.py:153-171): H_0 = X_0 (A_0 unused),
 * H_t = A_t H_{t-1} + X_t, independently for each of the R*N columns. */
ORC_EXPORT void orc_lin_fwd(const double* a, const double* x, double* h,
                            int64_t R, int64_t L, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < R; ++r) {
        const double* ar = a + r * L * N;
        const double* xr = x + r * L * N;
        double* hr = h + r * L * N;
        for (int64_t n = 0; n < N; ++n) hr[n] = xr[n];
        for (int64_t t = 1; t < L; ++t)
            for (int64_t n = 0; n < N; ++n)
                hr[t * N + n] = ar[t * N + n] * hr[(t - 1) * N + n] + xr[t * N + n];
    }
}

/* Gradient of orc_lin_fwd for loss = sum(H * g): gX_t = g_t + A_{t+1} gX_{t+1},
 * gA_t = gX_t H_{t-1} with gA_0 = 0 (the result PScan.backward, pscan.py:98-136,
 * is meant to return). */
ORC_EXPORT void orc_lin_bwd(const double* a, const double* h, const double* g,
                            double* ga, double* gx, int64_t R, int64_t L, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < R; ++r) {
        const double* ar = a + r * L * N;
        const double* hr = h + r * L * N;
        const double* gr = g + r * L * N;
        double* gar = ga + r * L * N;
        double* gxr = gx + r * L * N;
        for (int64_t n = 0; n < N; ++n) gxr[(L - 1) * N + n] = gr[(L - 1) * N + n];
        for (int64_t t = L - 2; t >= 0; --t)
            for (int64_t n = 0; n < N; ++n)
                gxr[t * N + n] = gr[t * N + n] + ar[(t + 1) * N + n] * gxr[(t + 1) * N + n];
        for (int64_t n = 0; n < N; ++n) gar[n] = 0.0;
        for (int64_t t = 1; t < L; ++t)
            for (int64_t n = 0; n < N; ++n)
                gar[t * N + n] = gxr[t * N + n] * hr[(t - 1) * N + n];
    }
}
