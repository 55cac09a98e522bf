/* blockscan_oracle.c -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Mamba-3 block scan ("Scan-B") of the reference MambaBlock:
 *   src/mamba_block.c:384-393  _ssm_scan_forward (1D: spatial_ndims <= 1)
 *   src/mamba_block.c:405-470  _ssm_scan_forward_callback (ND wavefront)
 * Per point t and state n (A = A_log used directly, no clamp in forward):
 *   a   = exp(dt_t * A[n]);  Bu = sum_r B[t, r*N+n] * u[t, r]
 *   ND: h = sum_K a * Rh(t-e_k)[n] + ((1-lam) dt / n_pred) * a * sum_K Bu(t-e_k)[n] + lam dt Bu
 *   1D: h = a * Rh(t-1)[n] + (1-lam) dt a * Bu(t-1)[n] + lam dt Bu
 *   y[t, r] = sum_n C[t, r*N+n] * h[n]
 * R rotates state pairs (2i, 2i+1) by theta[i] (odd last state unrotated).
 * Both forwards reproduce the reference's fp32 operation order.  The adjoint
 * is exact (double precision), not the reference's averaged-predecessor
 * approximation (src/mamba_block.c:640-695).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include "oracle.h"

#define MAXND 32

static float b_exp(float z, int fast) {
    if (!fast) return expf(z);
    if (z > 8.0f) z = 8.0f;
    if (z < -8.0f) z = -8.0f;
    return 1.0f + z + 0.5f * z * z + (1.0f / 6.0f) * z * z * z;
}
static double b_exp64(double z, int fast) {
    if (!fast) return exp(z);
    if (z > 8.0) z = 8.0;
    if (z < -8.0) z = -8.0;
    return 1.0 + z + 0.5 * z * z + (1.0 / 6.0) * z * z * z;
}
static double b_dexp64(double z, double e, int fast) {
    if (!fast) return e;
    if (z > 8.0 || z < -8.0) return 0.0;
    return 1.0 + z + 0.5 * z * z;
}

/* Reference src/mamba_block.c:384-393 (1D) and :405-470 (ND). */
int oracle_blockscan_fwd(const BlockScanArgs *a) {
    const long nd = a->ndims, N = a->N, R = a->R, NR = N * R;
    long L = 1, st[MAXND], idx[MAXND];
    if (nd < 0 || nd > MAXND || N <= 0 || R <= 0) return -1;
    for (long i = 0; i < nd; i++) L *= a->dims[i];
    if (nd == 0) L = a->L;
    { long s = 1; for (long i = nd - 1; i >= 0; i--) { st[i] = s; s *= a->dims[i]; } }
    if (nd <= 1) {
        float *hc = (float *)calloc(N, sizeof(float)), *hr = (float *)calloc(N, sizeof(float));
        float *pb = (float *)calloc(N, sizeof(float)), *bc = (float *)calloc(N, sizeof(float));
        for (long t = 0; t < L; t++) {
            float dt = a->dt[t], lam = a->lam ? a->lam[t] : a->default_lambda;
            const float *b = a->B + t * NR, *c = a->C + t * NR, *u = a->u + t * R;
            for (long i = 0; i + 1 < N; i += 2) {
                float th = a->theta[i >> 1], cv = cosf(th), sv = sinf(th), h0 = hc[i], h1 = hc[i + 1];
                hr[i] = cv * h0 - sv * h1;
                hr[i + 1] = sv * h0 + cv * h1;
            }
            if (N & 1) hr[N - 1] = hc[N - 1];
            memset(bc, 0, sizeof(float) * N);
            for (long r = 0; r < R; r++)
                for (long n = 0; n < N; n++) bc[n] += b[r * N + n] * u[r];
            memcpy(a->Bu + t * N, bc, sizeof(float) * N);
            for (long n = 0; n < N; n++) {
                float al = b_exp(dt * a->A[n], a->fast_exp);
                float beta = (1.0f - lam) * dt * al, gamma = lam * dt;
                hc[n] = al * hr[n] + beta * pb[n] + gamma * bc[n];
            }
            memcpy(a->h + t * N, hc, sizeof(float) * N);
            for (long r = 0; r < R; r++) {
                float yr = 0.0f;
                for (long n = 0; n < N; n++) yr += c[r * N + n] * hc[n];
                a->y[t * R + r] = yr;
            }
            memcpy(pb, bc, sizeof(float) * N);
        }
        free(hc); free(hr); free(pb); free(bc);
        return 0;
    }
    memset(a->h, 0, sizeof(float) * L * N);
    memset(a->Bu, 0, sizeof(float) * L * N);
    for (long t = 0; t < L; t++) {
        for (long i = 0; i < nd; i++) idx[i] = (t / st[i]) % a->dims[i];
        float dt = a->dt[t], lam = a->lam ? a->lam[t] : a->default_lambda;
        const float *b = a->B + t * NR, *c = a->C + t * NR, *u = a->u + t * R;
        for (long r = 0; r < R; r++) a->y[t * R + r] = 0.0f;
        for (long n = 0; n < N; n++) {
            float bu = 0.0f, hn = 0.0f, bacc = 0.0f;
            int np = 0;
            float al = b_exp(dt * a->A[n], a->fast_exp);
            for (long r = 0; r < R; r++) bu += b[r * N + n] * u[r];
            a->Bu[t * N + n] = bu;
            for (long ax = 0; ax < nd; ax++) {
                if (idx[ax] > 0) {
                    const float *hp = a->h + (t - st[ax]) * N;
                    float hrn;
                    if ((n & 1) && n > 0) {
                        float th = a->theta[n >> 1];
                        hrn = sinf(th) * hp[n - 1] + cosf(th) * hp[n];
                    } else if (n + 1 < N) {
                        float th = a->theta[n >> 1];
                        hrn = cosf(th) * hp[n] - sinf(th) * hp[n + 1];
                    } else {
                        hrn = hp[n];
                    }
                    hn += al * hrn;
                    bacc += a->Bu[(t - st[ax]) * N + n];
                    np++;
                }
            }
            if (np > 0) {
                float bs = (1.0f - lam) * dt / (float)np;
                hn += bs * al * bacc;
            }
            hn += lam * dt * bu;
            a->h[t * N + n] = hn;
            for (long r = 0; r < R; r++) a->y[t * R + r] += c[r * N + n] * hn;
        }
    }
    return 0;
}

/* Exact adjoint of the ND forward (the 1D forward is the same function).
 * Inputs: the forward arguments, saved h (a->h) and Bu (a->Bu), upstream
 * dy[L, R].  Outputs accumulated (+=) where non-NULL. */
int oracle_blockscan_bwd(const BlockScanArgs *a, const float *dy, BlockScanGrads *g) {
    const long nd = a->ndims < 1 ? 1 : a->ndims, N = a->N, R = a->R, NR = N * R;
    long L = 1, st[MAXND], idx[MAXND], dims[MAXND];
    if (a->ndims <= 0) { dims[0] = a->L; } else for (long i = 0; i < nd; i++) dims[i] = a->dims[i];
    for (long i = 0; i < nd; i++) L *= dims[i];
    { long s = 1; for (long i = nd - 1; i >= 0; i--) { st[i] = s; s *= dims[i]; } }
    double *ah = (double *)calloc((size_t)L * N, sizeof(double));
    double *ab = (double *)calloc((size_t)L * N, sizeof(double));
    double *gA = (double *)calloc(N, sizeof(double));
    double *gth = (double *)calloc(N / 2 + 1, sizeof(double));
    double *cs = (double *)malloc(sizeof(double) * (N / 2 + 1)), *sn = (double *)malloc(sizeof(double) * (N / 2 + 1));
    double *gh = (double *)malloc(sizeof(double) * N);
    if (!ah || !ab || !gA || !gth || !cs || !sn || !gh) return -1;
    for (long i = 0; i < N / 2; i++) { cs[i] = cos((double)a->theta[i]); sn[i] = sin((double)a->theta[i]); }
    for (long t = L - 1; t >= 0; t--) {
        for (long i = 0; i < nd; i++) idx[i] = (t / st[i]) % dims[i];
        const double dt = a->dt[t], lam = a->lam ? a->lam[t] : a->default_lambda;
        const float *b = a->B + t * NR, *c = a->C + t * NR, *u = a->u + t * R;
        /* g_h = C^T dy + R^T acc_hat ; dtheta from the rotation of h(t) */
        for (long n = 0; n < N; n++) {
            double v;
            const long n0 = n & ~1L;
            if (n0 + 1 < N) {
                const double a0 = ah[t * N + n0], a1 = ah[t * N + n0 + 1];
                const double cv = cs[n0 >> 1], sv = sn[n0 >> 1];
                v = (n & 1) ? (-sv * a0 + cv * a1) : (cv * a0 + sv * a1);
            } else {
                v = ah[t * N + n];
            }
            for (long r = 0; r < R; r++) v += (double)c[r * N + n] * dy[t * R + r];
            gh[n] = v;
        }
        for (long i = 0; i + 1 < N; i += 2) {
            double h0 = a->h[t * N + i], h1 = a->h[t * N + i + 1];
            double cv = cs[i >> 1], sv = sn[i >> 1];
            double hat0 = cv * h0 - sv * h1, hat1 = sv * h0 + cv * h1;
            gth[i >> 1] += -ah[t * N + i] * hat1 + ah[t * N + i + 1] * hat0;
        }
        int np = 0;
        for (long k = 0; k < nd; k++) np += idx[k] > 0;
        double gdt = 0.0, glam = 0.0;
        for (long n = 0; n < N; n++) {
            const double ghn = gh[n];
            if (g->dC) for (long r = 0; r < R; r++) g->dC[t * NR + r * N + n] += (float)(dy[t * R + r] * (double)a->h[t * N + n]);
            const double bu = a->Bu[t * N + n];
            const double gam = lam * dt;
            const double gbu = gam * ghn + ab[t * N + n];
            for (long r = 0; r < R; r++) {
                if (g->dB) g->dB[t * NR + r * N + n] += (float)(gbu * u[r]);
                if (g->du) g->du[t * R + r] += (float)(gbu * b[r * N + n]);
            }
            gdt += lam * bu * ghn;
            glam += dt * bu * ghn;
            if (np > 0) {
                const double A = a->A[n];
                const double z = dt * A;
                const double al = b_exp64(z, a->fast_exp);
                double sbu = 0.0, shat = 0.0;
                for (long k = 0; k < nd; k++) {
                    if (idx[k] == 0) continue;
                    long q = t - st[k];
                    sbu += a->Bu[q * N + n];
                    double hat;
                    long n0 = n & ~1L;
                    if (n0 + 1 < N) {
                        double h0 = a->h[q * N + n0], h1 = a->h[q * N + n0 + 1];
                        double cv = cs[n0 >> 1], sv = sn[n0 >> 1];
                        hat = (n & 1) ? sv * h0 + cv * h1 : cv * h0 - sv * h1;
                    } else {
                        hat = a->h[q * N + n];
                    }
                    shat += hat;
                    ah[q * N + n] += al * ghn;
                    ab[q * N + n] += (1.0 - lam) * dt / np * al * ghn;
                }
                const double s = (1.0 - lam) * dt / np;
                const double dal = shat * ghn + s * sbu * ghn;
                const double dz = b_dexp64(z, al, a->fast_exp) * dal;
                gdt += dz * A;
                gA[n] += dz * dt;
                const double ds = al * sbu * ghn;          /* d/ds */
                gdt += (1.0 - lam) / np * ds;
                glam += -dt / np * ds;
            }
        }
        if (g->ddt) g->ddt[t] += (float)gdt;
        if (g->dlam) g->dlam[t] += (float)glam;
    }
    if (g->dA) for (long n = 0; n < N; n++) g->dA[n] += (float)gA[n];
    if (g->dtheta) for (long i = 0; i < N / 2; i++) g->dtheta[i] += (float)gth[i];
    free(ah); free(ab); free(gA); free(gth); free(cs); free(sn); free(gh);
    return 0;
}

/* Double-precision Scan-B forward (ND formula; for finite differences).
 * Arrays as in BlockScanArgs but double. */
int oracle_blockscan_fwd64(long ndims, const long *dims, long N, long R, const double *u, const double *dt,
                           const double *lam, const double *B, const double *C, const double *A,
                           const double *theta, double default_lambda, int fast, double *h, double *y) {
    const long nd = ndims, NR = N * R;
    long L = 1, st[MAXND], idx[MAXND];
    for (long i = 0; i < nd; i++) L *= dims[i];
    { long s = 1; for (long i = nd - 1; i >= 0; i--) { st[i] = s; s *= dims[i]; } }
    double *Bu = (double *)calloc((size_t)L * N, sizeof(double));
    if (!Bu) return -1;
    for (long t = 0; t < L; t++) {
        for (long i = 0; i < nd; i++) idx[i] = (t / st[i]) % dims[i];
        const double d = dt[t], l = lam ? lam[t] : default_lambda;
        for (long r = 0; r < R; r++) y[t * R + r] = 0.0;
        for (long n = 0; n < N; n++) {
            double bu = 0.0, hn = 0.0, bacc = 0.0;
            int np = 0;
            const double al = b_exp64(d * A[n], fast);
            for (long r = 0; r < R; r++) bu += B[t * NR + r * N + n] * u[t * R + r];
            Bu[t * N + n] = bu;
            for (long ax = 0; ax < nd; ax++) {
                if (idx[ax] == 0) continue;
                const double *hp = h + (t - st[ax]) * N;
                const long n0 = n & ~1L;
                double hr;
                if (n0 + 1 < N) {
                    const double c = cos(theta[n0 >> 1]), s = sin(theta[n0 >> 1]);
                    hr = (n & 1) ? s * hp[n0] + c * hp[n0 + 1] : c * hp[n0] - s * hp[n0 + 1];
                } else {
                    hr = hp[n];
                }
                hn += al * hr;
                bacc += Bu[(t - st[ax]) * N + n];
                np++;
            }
            if (np > 0) hn += (1.0 - l) * d / np * al * bacc;
            hn += l * d * bu;
            h[t * N + n] = hn;
            for (long r = 0; r < R; r++) y[t * R + r] += C[t * NR + r * N + n] * hn;
        }
    }
    free(Bu);
    return 0;
}
