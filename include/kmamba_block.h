/* kmamba_block.h -- Mamba-3 block scan ("Scan-B") on the B200.
 *
 * The reference computes this scan inside the MambaBlock, in static functions
 * (src/mamba_block.c:384-470 forward, :530-744 backward), and its GPU block
 * path routes it through om_scannd_* with mismatched shapes
 * (cuda/mamba_block.cu:271-292).  These entry points expose the scan itself,
 * batched, on device buffers, with the reference's layouts:
 *   u[L,R], dt[L], lambda[L], B/C[L, R*N] (index r*N + n), A_log[N] (used as A),
 *   theta[N/2] (state pairs 2i, 2i+1), h/Bu[L,N], y[L,R]; per-item tensors are
 *   contiguous [batch, ...] blocks, A_log and theta are shared.
 * Forward (reference order of operations; 1D grids use the 1D recurrence):
 *   a = exp(dt A[n]);  Bu = sum_r B u;  h = sum_K a Rh(t-e_k) + ((1-lam) dt / n_pred) a sum_K Bu(t-e_k)
 *       + lam dt Bu;  y[t,r] = sum_n C h.
 * Backward: the exact adjoint of that forward (the reference's block backward
 * averages predecessors for ndims >= 2 and is not an exact gradient).
 * N <= 64.  Return 0 / -1 (kmb_last_error() has the reason).
 */
#ifndef KMB200_BLOCK_H
#define KMB200_BLOCK_H
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    long ndims;             /* grid rank (0 or 1 = 1D over L) */
    const long *dims;       /* host memory [ndims] */
    long L;                 /* points per item (product of dims) */
    long N, R;              /* states, MIMO rank */
    const float *u, *dt, *lambda, *B, *C, *A_log, *theta;
    float default_lambda;   /* used when lambda == NULL */
    int use_fast_exp;
    float *h, *Bu, *y;      /* forward outputs; read back by the backward */
} KMBlockScanParams;

typedef struct {
    float *dB, *dC;         /* [batch, L, R*N]  += */
    float *du;              /* [batch, L, R]    += */
    float *ddt, *dlambda;   /* [batch, L]       += */
    float *dA_log;          /* [N]    += summed over the batch */
    float *dtheta;          /* [N/2]  += summed over the batch */
} KMBlockScanGrads;

/* No counterpart in the reference API (see above): batched Scan-B forward. */
int kmb_blockscan_forward(const KMBlockScanParams *p, long batch, void *stream);
/* No counterpart in the reference API: exact Scan-B backward; dy is [batch, L, R]. */
int kmb_blockscan_backward(const KMBlockScanParams *p, long batch, const float *dy,
                           const KMBlockScanGrads *g, void *stream);

#ifdef __cplusplus
}
#endif
#endif
