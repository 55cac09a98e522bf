/* scan_nd.h -- public C ABI of the B200 scanND operator (k-mamba drop-in).
 *
 * The struct layout and function names are those of the reference interface
 * include/scan_nd.h:40-88 (goldensam777/BissiMamba), so an existing caller that
 * fills a ScanNDParams and calls scannd() links against libkmamba_b200.so
 * unchanged.  Field order/types are kept identical on purpose: the struct is
 * passed by pointer across the ABI.
 *
 * Layouts (row-major, P = prod(dims)):
 *   x[P,D]  A[ndims,D,M]  B,C,h[P,D,M]  delta[ndims,P,D]  y[P,D]
 *   theta[D/2] (channel pairs 2i,2i+1; odd last channel unrotated)  lambda[P]
 *
 * Recurrence (Scan-A, reference src/scan_nd.c:43-217), per point p, channel d,
 * state m, with K = axes where p has a predecessor p-e_k and n = |K|:
 *   a_k  = exp(delta_k[p,d] * A'_k[d,m])      A' = min(A, a_log_min) if clamped
 *   dt   = sum_{all axes} delta_k[p,d]
 *   beta = (1-lambda_p) * dt * (sum_K a_k)/n,  gamma = lambda_p * dt
 *   h    = (sum_K B x(p-e_k))/n * beta + B x(p) * gamma + sum_K a_k * R h(p-e_k)
 *   y    = sum_m C h
 */
#ifndef KMB200_SCAN_ND_H
#define KMB200_SCAN_ND_H

#include "wavefront_plan.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    long         max_ndims;
    long         max_state;
    int          use_fast_exp;   /* 0 = expf, 1 = clamped cubic Taylor polynomial */
    const long  *dims;           /* host memory, [ndims] */
    long         ndims;
    long         D;
    long         M;
    const float *x;
    const float *A;
    const float *B;
    const float *C;
    const float *delta;
    float       *h;
    float       *y;              /* forward: output y; backward: upstream dy (reference convention) */
    const float *theta;          /* [D/2] or NULL */
    const float *lambda;         /* [P] or NULL */
    float        default_lambda;
    int          use_a_log_clamp;
    float        a_log_min;
    float       *dA;             /* backward outputs, accumulated (+=); each may be NULL */
    float       *dB;
    float       *dC;
    float       *ddelta;
    float       *dlambda;
    float       *dtheta;
} ScanNDParams;

/* Reference include/scan_nd.h:72 (src/scan_nd.c:29-41): 1 = valid, 0 = invalid. */
int scannd_validate(const ScanNDParams *p);

/* Reference include/scan_nd.h:81 (src/scan_nd.c:234-252).  Forward scan on the
 * B200.  Data pointers may be all device pointers (computed in place) or all
 * host pointers (staged through a cached device workspace, h and y copied back).
 * Returns 0 on success, -1 on invalid arguments / mixed pointer kinds / CUDA
 * error.  There is no CPU fallback. */
int scannd(ScanNDParams *p);

/* Reference include/scan_nd.h:78 (src/scan_nd.c:43-217).  The plan is checked
 * against dims (as the reference does) and the scan then runs on the GPU. */
int scannd_ref_with_plan(ScanNDParams *p, const KMWavefrontPlan *plan);

/* Reference include/scan_nd.h:86 (cuda/scan_nd.cu:544-613).  Device pointers
 * only; host pointers return -1. */
int om_scannd_forward(ScanNDParams *p);

/* Reference include/scan_nd.h:87 (cuda/scan_nd.cu:615-680).  Device pointers
 * only.  Reads the saved states from p->h and the upstream gradient dy[P,D]
 * from p->y (the reference's convention, cuda/mamba_block.cu:375).  Computes
 * the exact adjoint of the forward above and ACCUMULATES (+=) into every
 * non-NULL gradient among dA, dB, dC, ddelta, dlambda, dtheta. */
int om_scannd_backward(ScanNDParams *p);

/* ---- additive extensions (no counterpart in the reference API) ---------- */

/* Batched forward: per-item tensors (x, B, C, delta, h, y, lambda) are
 * contiguous [batch, ...] blocks of the single-item layout; A and theta are
 * shared.  Same pointer rules as scannd(). */
int scannd_batched(ScanNDParams *p, long batch);

/* Batched backward (device pointers).  dB, dC, ddelta, dlambda are per item;
 * dA and dtheta are summed over the batch.  dx (may be NULL) receives the
 * gradient w.r.t. x, per item [batch, P, D], accumulated (+=). */
int scannd_backward_batched(ScanNDParams *p, long batch, float *dx);

/* Asynchronous device-pointer variants: enqueue on `stream` (a cudaStream_t,
 * NULL = legacy default stream) and return without synchronising. */
int scannd_forward_async(ScanNDParams *p, long batch, void *stream);
int scannd_backward_async(ScanNDParams *p, long batch, float *dx, void *stream);

/* Backward with a choice of output semantics (no counterpart in the reference,
 * whose GPU backward accumulates with atomicAdd, cuda/scan_nd.cu:367-537):
 * overwrite = 0 accumulates into dA, dB, dC, ddelta, dlambda, dtheta and dx
 * (+=, as scannd_backward_async); overwrite = 1 assigns them, so the caller
 * need not clear them and the 2D kernel does not read them back. */
int scannd_backward_ex(ScanNDParams *p, long batch, float *dx, int overwrite, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* KMB200_SCAN_ND_H */
