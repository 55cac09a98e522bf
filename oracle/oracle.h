/* oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatements of the reference algorithms, used by tests/, bench.py's
 * cpu_baseline leg and __graft_entry__.smoke() as the checker.  Nothing in the
 * product library (bissimamba_b200/) links or calls this code.
 *
 * Pinning: scannd/convnd forwards are checked bit-for-bit or within 1 ulp-level
 * tolerance against the reference compiled in place (oracle/_ref) and against
 * the reference's own known-answer vectors (tests/unit/test_scan_nd.c:63,121,
 * tests/unit/test_convnd_full.c:19).  The scannd backward has no trustworthy
 * reference (cuda/scan_nd.cu:367-537 is not the exact adjoint), so the
 * double-precision adjoint here is pinned by central finite differences of the
 * forward, which is itself pinned to the reference.
 */
#ifndef KMB_ORACLE_H
#define KMB_ORACLE_H
#include "../include/scan_nd.h"
#include "../include/convnd.h"

/* Scan-A forward, fp32, the reference's per-point operation order. */
int oracle_scannd_fwd(const ScanNDParams *p);

/* Scan-A forward in double (for finite differences).  Same layouts. */
int oracle_scannd_fwd_f64(const long *dims, long ndims, long D, long M,
                          const double *x, const double *A, const double *B,
                          const double *C, const double *delta,
                          const double *theta, const double *lambda,
                          double default_lambda, int use_a_log_clamp, double a_log_min,
                          int use_fast_exp, double *h, double *y);

/* Exact adjoint of Scan-A, computed in double from the fp32 inputs and saved
 * states p->h; dy is read from p->y.  Accumulates (+=) into the non-NULL
 * gradients of p and into dx[P,D] (may be NULL). */
int oracle_scannd_bwd(const ScanNDParams *p, float *dx);

/* Dense causal depthwise convND forward / backward, reference order. */
int oracle_convnd_fwd(const ConvNDParams *p);
int oracle_convnd_bwd(const ConvNDParams *p);

/* Mamba-3 block scan (Scan-B), one batch item.  B, C: [L, R*N] (index
 * r*N + n), u: [L, R], dt / lam: [L], A: [N] (A_log used as A), theta: [N/2].
 * ndims = 0 or 1 selects the reference's 1D recurrence, >= 2 the ND one. */
typedef struct {
    long ndims;
    const long *dims;
    long L;                 /* used when ndims == 0 */
    long N, R;
    const float *u, *dt, *lam, *B, *C, *A, *theta;
    float default_lambda;
    int fast_exp;
    float *h, *Bu, *y;      /* outputs [L,N], [L,N], [L,R] */
} BlockScanArgs;

typedef struct {
    float *dB, *dC, *du, *ddt, *dlam, *dA, *dtheta;
} BlockScanGrads;

int oracle_blockscan_fwd(const BlockScanArgs *a);
int oracle_blockscan_bwd(const BlockScanArgs *a, const float *dy, BlockScanGrads *g);
int oracle_blockscan_fwd64(long ndims, const long *dims, long N, long R, const double *u, const double *dt,
                           const double *lam, const double *B, const double *C, const double *A,
                           const double *theta, double default_lambda, int fast, double *h, double *y);

#endif
