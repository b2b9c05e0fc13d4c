/*
 * CPU oracle for the selective-scan hot path (TEST INFRASTRUCTURE ONLY).
 *
 * This file restates, in plain C and float64, the algorithms of the reference
 * (BhanuPrakash6640/SwiftX) for the selective scan, its backward pass, the
 * depthwise causal conv1d + SiLU that feeds it, and the recurrent decode step.
 * It is what the CUDA kernels are compared against.  Only the test
 * suite, the smoke check and the CPU-baseline leg of the benchmark load it;
 * the product library never links or calls it.
 *
 * Reference anchors (paths inside the reference project):
 *   models/selective_scan.py:34-60    selective_scan_ref  (forward recurrence)
 *   models/selective_scan.py:211-243  _FusedScanFn.backward (reverse recurrence)
 *   models/sift_block.py:108          delta = softplus(dt_proj(dt)), bias inside dt_proj
 *   models/sift_block.py:117-118      causal depthwise conv1d (pad d_conv-1, keep first L) + SiLU
 *   models/sift_block.py:134          y * silu(z) gate
 *   models/sift_block.py:153-175      SiftBlock.step (decode)
 *   models/selective_scan.py:91-99    sequential_scan (h_t = a_t * h_{t-1} + x_t loop)
 *
 * Layouts follow the reference API: u, delta, z, y are (b, L, D); B, C are
 * (b, L, N); A is (D, N); D-skip, delta_bias are (D,); states are (b, D, N);
 * the conv state is (b, D, K); all arrays are dense row-major.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define IDX3(i, j, k, J, K) (((size_t)(i) * (J) + (j)) * (K) + (k))

/* torch.nn.functional.softplus with beta=1, threshold=20. */
static double softplus(double x) { return x > 20.0 ? x : log1p(exp(x)); }
static double dsoftplus(double x) { return x > 20.0 ? 1.0 : 1.0 / (1.0 + exp(-x)); }
static double sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }
static double silu(double x) { return x * sigmoid(x); }
static double dsilu(double x) { double s = sigmoid(x); return s * (1.0 + x * (1.0 - s)); }

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* delta used by the recurrence: softplus(delta_raw + bias) or delta_raw + bias. */
static double eff_delta(double raw, const double* bias, int d, int use_softplus) {
    double v = raw + (bias ? bias[d] : 0.0);
    return use_softplus ? softplus(v) : v;
}

/*
 * Forward.  h_t = exp(delta_t*A) h_{t-1} + delta_t*u_t*B_t ;  y_t = <C_t, h_t> + Dskip*u_t ;
 * out_t = y_t * silu(z_t) when z is given, else y_t.
 * Follows selective_scan_ref (models/selective_scan.py:34-60) with the block's
 * softplus (sift_block.py:108) and gate (sift_block.py:134) glue.
 * h0 (optional) is the state before t=0; h_last (optional) receives h_{L-1};
 * ypre (optional) receives y before the gate.
 */
void orc_scan_fwd(int b, int L, int D, int N,
                  const double* u, const double* delta, const double* A,
                  const double* B, const double* C, const double* Dskip,
                  const double* z, const double* bias, int use_softplus,
                  const double* h0, double* out, double* ypre, double* h_last) {
    #pragma omp parallel for schedule(static)
    for (long bd = 0; bd < (long)b * D; ++bd) {
        int bi = (int)(bd / D), d = (int)(bd % D);
        double h[64];
        for (int n = 0; n < N; ++n) h[n] = h0 ? h0[IDX3(bi, d, n, D, N)] : 0.0;
        for (int t = 0; t < L; ++t) {
            size_t o = IDX3(bi, t, d, L, D);
            double dt = eff_delta(delta[o], bias, d, use_softplus);
            double ut = u[o], y = 0.0;
            for (int n = 0; n < N; ++n) {
                double a = exp(dt * A[(size_t)d * N + n]);
                h[n] = a * h[n] + dt * B[IDX3(bi, t, n, L, N)] * ut;
                y += h[n] * C[IDX3(bi, t, n, L, N)];
            }
            if (Dskip) y += ut * Dskip[d];
            if (ypre) ypre[o] = y;
            out[o] = z ? y * silu(z[o]) : y;
        }
        if (h_last)
            for (int n = 0; n < N; ++n) h_last[IDX3(bi, d, n, D, N)] = h[n];
    }
}

/*
 * Backward of orc_scan_fwd.  Follows _FusedScanFn.backward
 * (models/selective_scan.py:211-243): states are recomputed forward, then the
 * reverse recurrence  g_t = C_t*dy_t + exp(delta_{t+1}*A)*g_{t+1}  gives dL/dh_t and
 *   d delta += sum_n g*h_{t-1}*exp(delta*A)*A + u*sum_n g*B
 *   dA      += g*h_{t-1}*exp(delta*A)*delta
 *   dB_t    += g*delta*u   (summed over channels)
 *   dC_t    += dy*h_t      (summed over channels)
 *   du       = delta*sum_n g*B + Dskip*dy ;  dDskip += dy*u
 * The gate and softplus are chained on top (dz = dout*y*silu'(z), dy = dout*silu(z);
 * d delta_raw = d delta * softplus'(delta_raw + bias); dbias = sum d delta_raw).
 * Any output pointer may be NULL when not wanted (dD, dz, dbias, dh0).
 * Reductions are done per channel-block in fixed order, so results are deterministic.
 */
void orc_scan_bwd(int b, int L, int D, int N,
                  const double* u, const double* delta, const double* A,
                  const double* B, const double* C, const double* Dskip,
                  const double* z, const double* bias, int use_softplus,
                  const double* h0, const double* dout,
                  double* du, double* ddelta, double* dA, double* dB, double* dC,
                  double* dD, double* dz, double* dbias, double* dh0) {
    const int DB = 32;                         /* channels per work item */
    int nblk = (D + DB - 1) / DB;
    long items = (long)b * nblk;
    double* pB = (double*)calloc((size_t)items * L * N, sizeof(double));
    double* pC = (double*)calloc((size_t)items * L * N, sizeof(double));
    double* pA = (double*)calloc((size_t)b * D * N, sizeof(double));
    double* pD = (double*)calloc((size_t)b * D, sizeof(double));
    double* pbias = (double*)calloc((size_t)b * D, sizeof(double));

    #pragma omp parallel
    {
        double* hs = (double*)malloc((size_t)(L + 1) * N * sizeof(double));
        #pragma omp for schedule(dynamic)
        for (long it = 0; it < items; ++it) {
            int bi = (int)(it / nblk), blk = (int)(it % nblk);
            double* myB = pB + (size_t)it * L * N;
            double* myC = pC + (size_t)it * L * N;
            for (int d = blk * DB; d < D && d < (blk + 1) * DB; ++d) {
                const double* Ad = A + (size_t)d * N;
                /* recompute all states of this channel: hs[t+1] = h_t, hs[0] = h0 */
                for (int n = 0; n < N; ++n) hs[n] = h0 ? h0[IDX3(bi, d, n, D, N)] : 0.0;
                for (int t = 0; t < L; ++t) {
                    size_t o = IDX3(bi, t, d, L, D);
                    double dt = eff_delta(delta[o], bias, d, use_softplus);
                    for (int n = 0; n < N; ++n)
                        hs[(size_t)(t + 1) * N + n] = exp(dt * Ad[n]) * hs[(size_t)t * N + n]
                                                      + dt * B[IDX3(bi, t, n, L, N)] * u[o];
                }
                double g[64], accA[64];
                for (int n = 0; n < N; ++n) { g[n] = 0.0; accA[n] = 0.0; }
                double accD = 0.0, accbias = 0.0;
                for (int t = L - 1; t >= 0; --t) {
                    size_t o = IDX3(bi, t, d, L, D);
                    double raw = delta[o] + (bias ? bias[d] : 0.0);
                    double dt = use_softplus ? softplus(raw) : raw;
                    double ut = u[o];
                    const double* ht = hs + (size_t)(t + 1) * N;
                    const double* hp = hs + (size_t)t * N;
                    /* pre-gate output, needed for dz */
                    double y = 0.0;
                    for (int n = 0; n < N; ++n) y += ht[n] * C[IDX3(bi, t, n, L, N)];
                    if (Dskip) y += ut * Dskip[d];
                    double dy = dout[o];
                    if (z) {
                        if (dz) dz[o] = dout[o] * y * dsilu(z[o]);
                        dy = dout[o] * silu(z[o]);
                    }
                    double sgb = 0.0, sda = 0.0;
                    for (int n = 0; n < N; ++n) {
                        double Bn = B[IDX3(bi, t, n, L, N)], Cn = C[IDX3(bi, t, n, L, N)];
                        double a = exp(dt * Ad[n]);
                        myC[(size_t)t * N + n] += dy * ht[n];
                        g[n] += dy * Cn;                       /* total dL/dh_t */
                        double gpre = g[n] * hp[n] * a;         /* through exp(delta*A) */
                        sda += gpre * Ad[n];
                        accA[n] += gpre * dt;
                        sgb += g[n] * Bn;
                        myB[(size_t)t * N + n] += g[n] * dt * ut;
                        g[n] *= a;                              /* hand to h_{t-1} */
                    }
                    double gdelta = sda + sgb * ut;
                    du[o] = sgb * dt + (Dskip ? Dskip[d] * dy : 0.0);
                    double graw = use_softplus ? gdelta * dsoftplus(raw) : gdelta;
                    ddelta[o] = graw;
                    accbias += graw;
                    accD += dy * ut;
                }
                for (int n = 0; n < N; ++n) {
                    pA[IDX3(bi, d, n, D, N)] = accA[n];
                    if (dh0) dh0[IDX3(bi, d, n, D, N)] = g[n];
                }
                pD[(size_t)bi * D + d] = accD;
                pbias[(size_t)bi * D + d] = accbias;
            }
        }
        free(hs);
    }
    /* fixed-order reductions */
    #pragma omp parallel for schedule(static)
    for (long bt = 0; bt < (long)b * L; ++bt) {
        int bi = (int)(bt / L), t = (int)(bt % L);
        for (int n = 0; n < N; ++n) {
            double sb = 0.0, sc = 0.0;
            for (int blk = 0; blk < nblk; ++blk) {
                size_t base = ((size_t)bi * nblk + blk) * L * N + (size_t)t * N + n;
                sb += pB[base];
                sc += pC[base];
            }
            dB[IDX3(bi, t, n, L, N)] = sb;
            dC[IDX3(bi, t, n, L, N)] = sc;
        }
    }
    for (int d = 0; d < D; ++d) {
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int bi = 0; bi < b; ++bi) s += pA[IDX3(bi, d, n, D, N)];
            dA[(size_t)d * N + n] = s;
        }
        double sD = 0.0, sb = 0.0;
        for (int bi = 0; bi < b; ++bi) { sD += pD[(size_t)bi * D + d]; sb += pbias[(size_t)bi * D + d]; }
        if (dD) dD[d] = sD;
        if (dbias) dbias[d] = sb;
    }
    free(pB); free(pC); free(pA); free(pD); free(pbias);
}

/*
 * Causal depthwise conv1d + optional SiLU, as in models/sift_block.py:62-65,117-118:
 * nn.Conv1d(D, D, K, groups=D, padding=K-1) then keep the first L outputs, so
 *   pre_t = bias + sum_{k<K} w[d,k] * x_{t-(K-1)+k}   (x_s = 0 for s < 0)
 * x is addressed with element strides (sb, sl) and unit channel stride, so the
 * x half of the in_proj output (row stride 2D) can be passed as it is.
 */
void orc_conv1d_fwd(int b, int L, int D, int K, const double* x, long sb, long sl,
                    const double* w, const double* bias, int use_silu, double* out) {
    #pragma omp parallel for schedule(static)
    for (long bd = 0; bd < (long)b * D; ++bd) {
        int bi = (int)(bd / D), d = (int)(bd % D);
        for (int t = 0; t < L; ++t) {
            double s = bias ? bias[d] : 0.0;
            for (int k = 0; k < K; ++k) {
                int ts = t - (K - 1) + k;
                if (ts >= 0) s += w[(size_t)d * K + k] * x[bi * sb + ts * sl + d];
            }
            out[IDX3(bi, t, d, L, D)] = use_silu ? silu(s) : s;
        }
    }
}

/* Backward of orc_conv1d_fwd: dx (dense (b,L,D)), dw (D,K), dbias (D). */
void orc_conv1d_bwd(int b, int L, int D, int K, const double* x, long sb, long sl,
                    const double* w, const double* bias, int use_silu, const double* dout,
                    double* dx, double* dw, double* dbias) {
    #pragma omp parallel for schedule(static)
    for (int d = 0; d < D; ++d) {
        double accw[16] = {0}, accb = 0.0;
        for (int bi = 0; bi < b; ++bi) {
            for (int t = 0; t < L; ++t) dx[IDX3(bi, t, d, L, D)] = 0.0;
            for (int t = 0; t < L; ++t) {
                double s = bias ? bias[d] : 0.0;
                for (int k = 0; k < K; ++k) {
                    int ts = t - (K - 1) + k;
                    if (ts >= 0) s += w[(size_t)d * K + k] * x[bi * sb + ts * sl + d];
                }
                double gp = dout[IDX3(bi, t, d, L, D)] * (use_silu ? dsilu(s) : 1.0);
                accb += gp;
                for (int k = 0; k < K; ++k) {
                    int ts = t - (K - 1) + k;
                    if (ts >= 0) {
                        accw[k] += gp * x[bi * sb + ts * sl + d];
                        dx[IDX3(bi, ts, d, L, D)] += gp * w[(size_t)d * K + k];
                    }
                }
            }
        }
        for (int k = 0; k < K; ++k) dw[(size_t)d * K + k] = accw[k];
        if (dbias) dbias[d] = accb;
    }
}

/*
 * One recurrent decode step, following SiftBlock.step (models/sift_block.py:153-175)
 * with delta_raw, B and C given (they come from x_proj/dt_proj in the block):
 *   conv_state <- roll left by one, append x ; xc = silu(<conv_state, w> + conv_bias)
 *   delta = softplus(delta_raw + dt_bias) (or delta_raw + dt_bias)
 *   ssm_state <- exp(delta*A)*ssm_state + delta*B*xc ;  y = <ssm_state, C> + Dskip*xc
 *   out = y * silu(z)  (z optional) ;  xc_out (optional) receives xc.
 * conv_state (b,D,K) and ssm_state (b,D,N) are updated in place.
 */
void orc_decode_step(int b, int D, int N, int K, const double* x, const double* z,
                     const double* delta_raw, const double* B, const double* C,
                     const double* conv_w, const double* conv_b, const double* A,
                     const double* Dskip, const double* dt_bias, int use_softplus,
                     double* conv_state, double* ssm_state, double* out, double* xc_out) {
    #pragma omp parallel for schedule(static)
    for (long bd = 0; bd < (long)b * D; ++bd) {
        int bi = (int)(bd / D), d = (int)(bd % D);
        double* cs = conv_state + IDX3(bi, d, 0, D, K);
        for (int k = 0; k < K - 1; ++k) cs[k] = cs[k + 1];
        cs[K - 1] = x[(size_t)bi * D + d];
        double s = conv_b ? conv_b[d] : 0.0;
        for (int k = 0; k < K; ++k) s += cs[k] * conv_w[(size_t)d * K + k];
        double xc = silu(s);
        if (xc_out) xc_out[(size_t)bi * D + d] = xc;
        double dt = eff_delta(delta_raw[(size_t)bi * D + d], dt_bias, d, use_softplus);
        double y = 0.0;
        double* h = ssm_state + IDX3(bi, d, 0, D, N);
        for (int n = 0; n < N; ++n) {
            double a = exp(dt * A[(size_t)d * N + n]);
            h[n] = h[n] * a + dt * B[(size_t)bi * N + n] * xc;
            y += h[n] * C[(size_t)bi * N + n];
        }
        if (Dskip) y += Dskip[d] * xc;
        out[(size_t)bi * D + d] = z ? y * silu(z[(size_t)bi * D + d]) : y;
    }
}

/* sequential_scan (models/selective_scan.py:91-99): h = a[:, t] * h + x[:, t] along dim 1,
 * h starting at 0; a, x, h dense (b, L, W) with W the product of the trailing dims. */
void orc_linear_scan(int b, int L, long W, const double* a, const double* x, double* h) {
    #pragma omp parallel for schedule(static)
    for (long q = 0; q < (long)b * W; ++q) {
        const long bi = q / W, m = q % W;
        double acc = 0.0;
        for (int t = 0; t < L; ++t) {
            const size_t i = ((size_t)bi * L + t) * W + m;
            acc = a[i] * acc + x[i];
            h[i] = acc;
        }
    }
}

/* Adjoint of orc_linear_scan given the upstream gradient dh of h: g_t = dh_t + a_{t+1} g_{t+1}
 * (walked from the last step), dx_t = g_t, da_t = g_t * h_{t-1} with h_{-1} = 0. */
void orc_linear_scan_bwd(int b, int L, long W, const double* a, const double* h, const double* dh,
                         double* da, double* dx) {
    #pragma omp parallel for schedule(static)
    for (long q = 0; q < (long)b * W; ++q) {
        const long bi = q / W, m = q % W;
        double g = 0.0, an = 0.0;
        for (int t = L - 1; t >= 0; --t) {
            const size_t i = ((size_t)bi * L + t) * W + m;
            g = dh[i] + an * g;
            dx[i] = g;
            da[i] = t > 0 ? g * h[i - W] : 0.0;
            an = a[i];
        }
    }
}
