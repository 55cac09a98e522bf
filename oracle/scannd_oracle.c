/* scannd_oracle.c -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates the reference Scan-A forward of src/scan_nd.c:43-217 and derives its
 * exact adjoint.  Points are visited in row-major order, which is a causal
 * order (every predecessor p - stride[k] precedes p); the reference visits the
 * same points level by level (src/scan_nd.c:89-103), and because each point's
 * arithmetic only reads its predecessors the results are identical.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include "oracle.h"

#define MAXND 32

static long o_points(const long *dims, long nd) {
    long p = 1;
    for (long i = 0; i < nd; i++) p *= dims[i];
    return p;
}

static void o_strides(const long *dims, long nd, long *st) {
    long s = 1;
    for (long a = nd - 1; a >= 0; a--) { st[a] = s; s *= dims[a]; }
}

static void o_unravel(long off, const long *dims, const long *st, long nd, long *idx) {
    for (long a = 0; a < nd; a++) { idx[a] = (off / st[a]) % dims[a]; }
}

/* km_scan_exp, reference include/km_topology.h:52-60 (clamped cubic Taylor
 * polynomial when use_fast_exp, else libm expf). */
static float o_exp(float z, int fast) {
    if (!fast) return expf(z);
    if (z > 8.0f) z = 8.0f;
    if (z < -8.0f) z = -8.0f;
    return 1.0f + z + 0.5f * z * z + (1.0f / 6.0f) * z * z * z;
}
static double o_exp64(double z, int fast) {
    if (!fast) return exp(z);
    if (z > 8.0) z = 8.0;
    if (z < -8.0) z = -8.0;
    return 1.0 + z + 0.5 * z * z + (1.0 / 6.0) * z * z * z;
}
/* d/dz of o_exp64 */
static double o_dexp64(double z, double e, int fast) {
    if (!fast) return e;
    if (z > 8.0 || z < -8.0) return 0.0;
    return 1.0 + z + 0.5 * z * z;
}

static int o_valid(const ScanNDParams *p) {
    if (!p || !p->dims || p->ndims <= 0 || p->ndims > MAXND || p->D <= 0 || p->M <= 0) return 0;
    if (!p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->y) return 0;
    for (long a = 0; a < p->ndims; a++) if (p->dims[a] <= 0) return 0;
    return 1;
}

/* Reference src/scan_nd.c:103-201, one point at a time. */
int oracle_scannd_fwd(const ScanNDParams *p) {
    if (!o_valid(p)) return -1;
    const long nd = p->ndims, D = p->D, M = p->M;
    const long P = o_points(p->dims, nd);
    long st[MAXND], idx[MAXND];
    o_strides(p->dims, nd, st);
    /* Bu of every point (reference Bu_prev[P*D*M], src/scan_nd.c:71,171) and the
     * rotated states (reference h_rot, correctly sized here). */
    float *bu = (float *)calloc((size_t)P * D * M, sizeof(float));
    float *hr = p->theta ? (float *)calloc((size_t)P * D * M, sizeof(float)) : NULL;
    if (!bu || (p->theta && !hr)) { free(bu); free(hr); return -1; }

    for (long off = 0; off < P; off++) {
        o_unravel(off, p->dims, st, nd, idx);
        float lam = p->lambda ? p->lambda[off] : p->default_lambda;
        for (long d = 0; d < D; d++) {
            float xv = p->x[off * D + d];
            float dt = 0.0f, yacc = 0.0f;
            for (long a = 0; a < nd; a++) dt += p->delta[(a * P + off) * D + d];
            for (long m = 0; m < M; m++) {
                long dm = d * M + m, pdm = off * D * M + dm;
                float but = p->B[pdm] * xv;
                float buacc = 0.0f, dacc = 0.0f, hacc = 0.0f;
                int n = 0;
                for (long a = 0; a < nd; a++) {
                    if (idx[a] > 0) {
                        long q = (off - st[a]) * D * M + dm;
                        float dta = p->delta[(a * P + off) * D + d];
                        float av = p->A[(a * D + d) * M + m];
                        if (p->use_a_log_clamp && av > p->a_log_min) av = p->a_log_min;
                        float al = o_exp(dta * av, p->use_fast_exp);
                        buacc += bu[q];
                        dacc += al;
                        float hp = hr ? hr[q] : p->h[q];
                        hacc += al * hp;
                        n++;
                    }
                }
                float buavg = n > 0 ? buacc / n : 0.0f;
                float alavg = n > 0 ? dacc / n : 0.0f;
                float beta = (1.0f - lam) * dt * alavg;
                float gamma = lam * dt;
                float hn = buavg * beta + but * gamma + hacc;
                bu[pdm] = but;
                p->h[pdm] = hn;
                yacc += p->C[pdm] * hn;
            }
            p->y[off * D + d] = yacc;
        }
        if (hr) {
            for (long d = 0; d + 1 < D; d += 2) {
                float th = p->theta[d >> 1];
                float c = cosf(th), s = sinf(th);
                for (long m = 0; m < M; m++) {
                    long i0 = off * D * M + d * M + m, i1 = i0 + M;
                    float h0 = p->h[i0], h1 = p->h[i1];
                    hr[i0] = c * h0 - s * h1;
                    hr[i1] = s * h0 + c * h1;
                }
            }
            if (D & 1)
                for (long m = 0; m < M; m++) {
                    long i = off * D * M + (D - 1) * M + m;
                    hr[i] = p->h[i];
                }
        }
    }
    free(bu);
    free(hr);
    return 0;
}

/* Rotated state of point q (flat q*D*M base) for channel d, state m. */
static double o_hat64(const double *h, long base, long D, long M, long d, long m,
                      const double *cs, const double *sn) {
    if (!cs) return h[base + d * M + m];
    if ((D & 1) && d == D - 1) return h[base + d * M + m];
    long d0 = d & ~1L;
    double h0 = h[base + d0 * M + m], h1 = h[base + (d0 + 1) * M + m];
    double c = cs[d0 >> 1], s = sn[d0 >> 1];
    return (d & 1) ? s * h0 + c * h1 : c * h0 - s * h1;
}

/* |R| h for the magnitude bound (all entries non-negative). */
static double o_hatabs64(const double *h, long base, long D, long M, long d, long m,
                         const double *cs, const double *sn) {
    if (!cs) return h[base + d * M + m];
    if ((D & 1) && d == D - 1) return h[base + d * M + m];
    long d0 = d & ~1L;
    double h0 = h[base + d0 * M + m], h1 = h[base + (d0 + 1) * M + m];
    return cs[d0 >> 1] * ((d & 1) ? h1 : h0) + sn[d0 >> 1] * ((d & 1) ? h0 : h1);
}

int oracle_scannd_fwd_f64(const long *dims, long nd, long D, long M,
                          const double *x, const double *A, const double *B,
                          const double *C, const double *delta,
                          const double *theta, const double *lambda,
                          double default_lambda, int clamp, double a_log_min,
                          int fast, double *h, double *y) {
    if (!dims || nd <= 0 || nd > MAXND || D <= 0 || M <= 0) return -1;
    const long P = o_points(dims, nd);
    long st[MAXND], idx[MAXND];
    o_strides(dims, nd, st);
    double *cs = NULL, *sn = NULL;
    if (theta) {
        cs = (double *)malloc(sizeof(double) * (D / 2 + 1));
        sn = (double *)malloc(sizeof(double) * (D / 2 + 1));
        for (long i = 0; i < D / 2; i++) { cs[i] = cos(theta[i]); sn[i] = sin(theta[i]); }
    }
    for (long off = 0; off < P; off++) {
        o_unravel(off, dims, st, nd, idx);
        double lam = lambda ? lambda[off] : default_lambda;
        for (long d = 0; d < D; d++) {
            double xv = x[off * D + d], dt = 0.0, yacc = 0.0;
            for (long a = 0; a < nd; a++) dt += delta[(a * P + off) * D + d];
            for (long m = 0; m < M; m++) {
                long pdm = off * D * M + d * M + m;
                double but = B[pdm] * xv, buacc = 0, dacc = 0, hacc = 0;
                int n = 0;
                for (long a = 0; a < nd; a++) {
                    if (idx[a] > 0) {
                        long q = off - st[a];
                        double av = A[(a * D + d) * M + m];
                        if (clamp && av > a_log_min) av = a_log_min;
                        double al = o_exp64(delta[(a * P + off) * D + d] * av, fast);
                        buacc += B[q * D * M + d * M + m] * x[q * D + d];
                        dacc += al;
                        hacc += al * o_hat64(h, q * D * M, D, M, d, m, cs, sn);
                        n++;
                    }
                }
                double hn = but * lam * dt + hacc;
                if (n > 0) hn += (buacc / n) * (1.0 - lam) * dt * (dacc / n);
                h[pdm] = hn;
                yacc += C[pdm] * hn;
            }
            y[off * D + d] = yacc;
        }
    }
    free(cs);
    free(sn);
    return 0;
}

/* Exact adjoint.  With g_h(p) the total derivative of L = sum dy*y w.r.t. h(p):
 *   g_h(p)   = C dy + R^T sum_{s=p+e_k} a_k(s) g_h(s)
 *   g_Bu(p)  = gamma(p) g_h(p) + sum_{s=p+e_k} beta(s)/n(s) g_h(s)
 * accumulated by pushing from s to its predecessors while visiting points in
 * reverse row-major order. */
int oracle_scannd_bwd(const ScanNDParams *p, float *dx) {
    if (!o_valid(p)) return -1;
    const long nd = p->ndims, D = p->D, M = p->M;
    const long P = o_points(p->dims, nd);
    const long DM = D * M;
    long st[MAXND], idx[MAXND];
    o_strides(p->dims, nd, st);
    double *acc_hat = (double *)calloc((size_t)P * DM, sizeof(double));
    double *acc_bu = (double *)calloc((size_t)P * DM, sizeof(double));
    double *hd = (double *)malloc(sizeof(double) * (size_t)P * DM);
    double *gA = (double *)calloc((size_t)nd * DM, sizeof(double));
    double *gth = (double *)calloc((size_t)(D / 2 + 1), sizeof(double));
    double *cs = NULL, *sn = NULL;
    if (!acc_hat || !acc_bu || !hd || !gA || !gth) goto fail;
    for (long i = 0; i < P * DM; i++) hd[i] = p->h[i];
    if (p->theta) {
        cs = (double *)malloc(sizeof(double) * (D / 2 + 1));
        sn = (double *)malloc(sizeof(double) * (D / 2 + 1));
        for (long i = 0; i < D / 2; i++) { cs[i] = cos((double)p->theta[i]); sn[i] = sin((double)p->theta[i]); }
    }

    for (long off = P - 1; off >= 0; off--) {
        o_unravel(off, p->dims, st, nd, idx);
        const double lam = p->lambda ? p->lambda[off] : p->default_lambda;
        double glam = 0.0;
        const long base = off * DM;
        /* g_h for every (d,m) of this point: R^T applied to acc_hat. */
        for (long d = 0; d < D; d++) {
            const double dyv = p->y[off * D + d];
            const double xv = p->x[off * D + d];
            double dt = 0.0, gdt = 0.0, gx = 0.0;
            for (long a = 0; a < nd; a++) dt += p->delta[(a * P + off) * D + d];
            double gdel[MAXND];
            for (long a = 0; a < nd; a++) gdel[a] = 0.0;
            for (long m = 0; m < M; m++) {
                const long pdm = base + d * M + m;
                double gh;
                if (cs && !((D & 1) && d == D - 1)) {
                    long d0 = d & ~1L;
                    double a0 = acc_hat[base + d0 * M + m], a1 = acc_hat[base + (d0 + 1) * M + m];
                    double c = cs[d0 >> 1], s = sn[d0 >> 1];
                    gh = (d & 1) ? (-s * a0 + c * a1) : (c * a0 + s * a1);
                    if (!(d & 1)) {
                        /* d theta: g_hat . d(hat)/d theta, hat = R h(p) */
                        double h0 = hd[base + d0 * M + m], h1 = hd[base + (d0 + 1) * M + m];
                        double hat0 = c * h0 - s * h1, hat1 = s * h0 + c * h1;
                        gth[d0 >> 1] += -a0 * hat1 + a1 * hat0;
                    }
                } else {
                    gh = acc_hat[pdm];
                }
                gh += (double)p->C[pdm] * dyv;
                if (p->dC) p->dC[pdm] += (float)(dyv * hd[pdm]);

                const double bv = p->B[pdm];
                const double but = bv * xv;
                const double gamma = lam * dt;
                const double gbu = gamma * gh + acc_bu[pdm];
                if (p->dB) p->dB[pdm] += (float)(gbu * xv);
                gx += gbu * bv;
                /* gamma = lam*dt */
                double g_gamma = but * gh;
                gdt += lam * g_gamma;
                glam += dt * g_gamma;

                /* recompute the predecessor terms */
                double al[MAXND], avv[MAXND], dta[MAXND];
                int has[MAXND];
                double sbu = 0.0, sal = 0.0;
                int n = 0;
                for (long a = 0; a < nd; a++) {
                    has[a] = idx[a] > 0;
                    if (!has[a]) continue;
                    long q = off - st[a];
                    double av = p->A[(a * D + d) * M + m];
                    int clamped = p->use_a_log_clamp && av > p->a_log_min;
                    if (clamped) av = p->a_log_min;
                    avv[a] = clamped ? NAN : av; /* NAN marks "no gradient to A" */
                    dta[a] = p->delta[(a * P + off) * D + d];
                    al[a] = o_exp64(dta[a] * av, p->use_fast_exp);
                    sbu += (double)p->B[q * DM + d * M + m] * (double)p->x[q * D + d];
                    sal += al[a];
                    n++;
                }
                if (n > 0) {
                    const double beta = (1.0 - lam) * dt * (sal / n);
                    const double g_beta = (sbu / n) * gh;
                    const double g_sal = (1.0 - lam) * dt / n * g_beta;
                    gdt += (1.0 - lam) * (sal / n) * g_beta;
                    glam += -dt * (sal / n) * g_beta;
                    for (long a = 0; a < nd; a++) {
                        if (!has[a]) continue;
                        long q = off - st[a];
                        long qdm = q * DM + d * M + m;
                        double hat = o_hat64(hd, q * DM, D, M, d, m, cs, sn);
                        double gal = hat * gh + g_sal;
                        double av = isnan(avv[a]) ? p->a_log_min : avv[a];
                        double z = dta[a] * av;
                        double dz = o_dexp64(z, al[a], p->use_fast_exp) * gal;
                        gdel[a] += dz * av;
                        if (!isnan(avv[a])) gA[(a * D + d) * M + m] += dz * dta[a];
                        acc_hat[qdm] += al[a] * gh;
                        acc_bu[qdm] += beta / n * gh;
                    }
                }
            }
            if (p->ddelta)
                for (long a = 0; a < nd; a++)
                    p->ddelta[(a * P + off) * D + d] += (float)(gdel[a] + gdt);
            if (dx) dx[off * D + d] += (float)gx;
        }
        if (p->dlambda) p->dlambda[off] += (float)glam;
    }
    if (p->dA) for (long i = 0; i < nd * DM; i++) p->dA[i] += (float)gA[i];
    if (p->dtheta && p->theta) for (long i = 0; i < D / 2; i++) p->dtheta[i] += (float)gth[i];
    free(acc_hat); free(acc_bu); free(hd); free(gA); free(gth); free(cs); free(sn);
    return 0;
fail:
    free(acc_hat); free(acc_bu); free(hd); free(gA); free(gth);
    return -1;
}

/* Magnitude bound of the forward: the same recurrence evaluated in double on
 * absolute values (|x|, |B|, |C|, |cos|, |sin|; alpha, beta, gamma >= 0 for
 * lambda in [0,1]).  Hb(p) bounds the sum of the absolute values of every
 * term that contributes to h(p), so fp32 rounding in any evaluation order is
 * O(eps * Hb); the parity tests scale their tolerance by it. */
int oracle_scannd_bound(const ScanNDParams *p, double *Hb, double *Yb) {
    if (!o_valid(p)) return -1;
    const long nd = p->ndims, D = p->D, M = p->M;
    const long P = o_points(p->dims, nd);
    long st[MAXND], idx[MAXND];
    o_strides(p->dims, nd, st);
    double *cs = NULL, *sn = NULL;
    if (p->theta) {
        cs = (double *)malloc(sizeof(double) * (D / 2 + 1));
        sn = (double *)malloc(sizeof(double) * (D / 2 + 1));
        for (long i = 0; i < D / 2; i++) { cs[i] = fabs(cos((double)p->theta[i])); sn[i] = fabs(sin((double)p->theta[i])); }
    }
    for (long off = 0; off < P; off++) {
        o_unravel(off, p->dims, st, nd, idx);
        double lam = p->lambda ? p->lambda[off] : p->default_lambda;
        double lam1 = fabs(1.0 - lam);
        lam = fabs(lam);
        for (long d = 0; d < D; d++) {
            double xv = fabs(p->x[off * D + d]), dt = 0.0, yacc = 0.0;
            for (long a = 0; a < nd; a++) dt += fabs(p->delta[(a * P + off) * D + d]);
            for (long m = 0; m < M; m++) {
                long pdm = off * D * M + d * M + m;
                double but = fabs(p->B[pdm]) * xv, buacc = 0, dacc = 0, hacc = 0;
                int n = 0;
                for (long a = 0; a < nd; a++) {
                    if (idx[a] > 0) {
                        long q = off - st[a];
                        double av = p->A[(a * D + d) * M + m];
                        if (p->use_a_log_clamp && av > p->a_log_min) av = p->a_log_min;
                        double al = fabs(o_exp64(p->delta[(a * P + off) * D + d] * av, p->use_fast_exp));
                        buacc += fabs(p->B[q * D * M + d * M + m]) * fabs(p->x[q * D + d]);
                        dacc += al;
                        hacc += al * o_hatabs64(Hb, q * D * M, D, M, d, m, cs, sn);
                        n++;
                    }
                }
                double hn = but * lam * dt + hacc;
                if (n > 0) hn += (buacc / n) * lam1 * dt * (dacc / n);
                Hb[pdm] = hn;
                yacc += fabs(p->C[pdm]) * hn;
            }
            Yb[off * D + d] = yacc;
        }
    }
    free(cs);
    free(sn);
    return 0;
}
