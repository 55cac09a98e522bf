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
    int inputs_bf16;        /* 1: u, dt, lambda, B, C are bf16 arrays (state and outputs stay fp32) */
} KMBlockScanParams;

typedef struct {
    float *dB, *dC;         /* [batch, L, R*N]  += */
    float *du;              /* [batch, L, R]    += */
    float *ddt, *dlambda;   /* [batch, L]       += */
    float *dA_log;          /* [N]    += summed over the batch */
    float *dtheta;          /* [N/2]  += summed over the batch */
} KMBlockScanGrads;

/* Forward kernel choice, per host thread (for tests and comparison).  mode 1
 * (default): 2D grids with N even, R in {1, 2, 4} whose column strips fit in 8
 * warps use the grouped systolic strip kernel (the state pairs split over
 * several CTAs per item); other 2D grids with an inner extent <= 64, N <= 64,
 * R in {1, 2, 4} use the one-CTA-per-item strip kernel, with rows staged
 * through shared memory by bulk copies when the inner extent and N are
 * multiples of 8; 3: skip the grouped kernel; 2: the one-CTA-per-item strip
 * kernel always loads rows directly; 0: always the level-synchronous kernels.
 * The last forward's path: 3 grouped strips, 2 staged strips, 1 strips, 0 level
 * kernels, -1 none yet. */
void kmb_blockscan_set_strips(int mode);
int kmb_blockscan_last_forward_path(void);
/* Backward kernel choice, per host thread: on (default) 2D grids with R in
 * {1, 2, 4} whose column strips fit in 8 warps use the systolic strip backward;
 * off: always the level-synchronous kernels.  The last backward's path: 1
 * strips, 0 level kernels, -1 none yet. */
void kmb_blockscan_set_backward_strips(int on);
int kmb_blockscan_last_backward_path(void);
/* No counterpart in the reference API (see above): batched Scan-B forward. */
int kmb_blockscan_forward(const KMBlockScanParams *p, long batch, void *stream);
/* No counterpart in the reference API: exact Scan-B backward; dy is [batch, L, R]. */
int kmb_blockscan_backward(const KMBlockScanParams *p, long batch, const float *dy,
                           const KMBlockScanGrads *g, void *stream);
/* No counterpart in the reference API: the same backward; overwrite = 1 assigns
 * dB, dC, du, ddt and dlambda instead of accumulating into them (dA_log and
 * dtheta still accumulate), so the caller need not clear them first. */
int kmb_blockscan_backward_ex(const KMBlockScanParams *p, long batch, const float *dy,
                              const KMBlockScanGrads *g, int overwrite, void *stream);

/* ---- Mamba-3 block (reference MambaBlock, src/mamba_block.c:106-125,509-528,746-773;
 * GPU counterpart cuda/mamba_block.cu:223-415), batched, device pointers ---------- */
typedef struct {
    long dim, N, R;          /* model dim, state size, MIMO rank */
    long ndims;              /* spatial grid rank (0/1 = 1D over L) */
    const long *dims;        /* host memory */
    long L;                  /* points per item */
    float dt_min, dt_max, default_lambda;
    int use_fast_exp;
    int bf16_storage;        /* 1: x, out, dout, dx and the stored scan inputs are bf16;
                                projections run as bf16 x bf16 -> fp32 GEMMs; state, parameters
                                and their gradients stay fp32 (no counterpart in the reference,
                                whose use_bf16 flag is never read, include/kmamba.h:47-48) */
} KMBlockConfig;

/* Parameters, reference layouts (include/kmamba.h:152-175): W_in[R,dim],
 * W_out[dim,R], A_log[N], W_B/W_C[N*R,dim], delta_proj[dim], lambda_proj[dim],
 * b_B/b_C[N*R], theta[N/2].  The gradient struct has the same fields (+=). */
typedef struct {
    const float *W_in, *W_out, *A_log, *W_B, *W_C, *delta_proj, *lambda_proj, *b_B, *b_C, *theta;
} KMBlockWeights;
typedef struct {
    float *W_in, *W_out, *A_log, *W_B, *W_C, *delta_proj, *lambda_proj, *b_B, *b_C, *theta;
} KMBlockGrads;

/* Floats of the activation buffer the forward fills and the backward reads. */
size_t kmb_block_activation_floats(const KMBlockConfig *c, long batch);

/* Reference mamba_block_forward_ws (src/mamba_block.c:509-528) for `batch`
 * items: x, out [batch, L, dim].  u = silu(W_in x), dt = clamp(softplus(
 * delta_proj.x), dt_min, dt_max), lambda = sigmoid(lambda_proj.x), B = W_B x + b_B,
 * C = W_C x + b_C, block scan, out = x + W_out y.  Projections run on the
 * tensor cores at fp32 accuracy (split-bf16 pieces, fp32 accumulation; see
 * kmamba_gemm.h).  act: kmb_block_activation_floats() floats. */
/* bf16 storage: 1 (default) = block projections on the tensor cores with the
 * input epilogue fused (tcgen05); 0 = the plain tensor-core GEMM and separate
 * epilogues.
 * Per host thread; for comparison and tests. */
void kmb_block_set_tensor_cores(int on);
/* Projection used by this thread's last bf16 block forward: 1 = tensor cores,
 * 0 = plain GEMM + epilogue, -1 = none yet. */
int kmb_block_last_projection_path(void);
/* dx GEMM of this thread's last bf16 block backward: 1 = tensor cores (residual
 * fused), 0 = plain GEMM + residual kernel, -1 = none yet. */
int kmb_block_last_dx_path(void);
int kmb_block_forward(const KMBlockConfig *c, const KMBlockWeights *w, const float *x, float *out,
                      long batch, float *act, void *stream);

/* Exact gradient of kmb_block_forward: parameter gradients accumulate (+=)
 * into g (any field may be NULL); dx (may be NULL) receives the full input
 * gradient, including the W_in / W_B / W_C / delta / lambda paths that the
 * reference omits (src/mamba_block.c:772, d_input = dY). */
int kmb_block_backward(const KMBlockConfig *c, const KMBlockWeights *w, const float *x, const float *dout,
                       float *dx, const KMBlockGrads *g, long batch, const float *act, void *stream);

/* ---- the reference's GPU block entry points, same argument lists -------------
 * cuda/mamba_block.cu:223-244 and :306-346 (the prototype of the definition;
 * src/kmamba.c:36-51 declares a different argument order for the backward --
 * this one follows the definition).  All pointers are device pointers for one
 * sequence of L points; `cublas` is accepted and ignored.  The reference's GPU
 * block has no B / C biases, so none are applied.  The caller's workspace
 * buffers receive what the reference stores in them (u_raw, u, dt_raw, dt,
 * B_exp, C_exp, h_store, y_scan, y_proj, lambda_raw, lambda).  dt_exp may be
 * NULL, as the reference passes it; when given ([L, state] floats) it receives
 * the B*u products, and the backward reads them instead of recomputing them.
 * The backward accumulates the exact gradients (+=) and writes d_dx; its
 * scratch arguments (dy_scan .. dlambda_raw) are unused and may be NULL.
 * The computation is the CPU MambaBlock's (src/mamba_block.c), the same as
 * kmb_block_forward with zero B / C biases, dt in [1e-3, 0.1] and default
 * lambda 0.5.  The reference's GPU body instead runs the Scan-A kernel with
 * D = state, M = 1 over u[L, R] (cuda/mamba_block.cu:271-291), which reads past
 * u whenever state > R; that is not reproduced.  d_dx may alias d_dy, as the
 * reference model passes it (src/kmamba.c:567-568).
 * There is no error channel in these void functions: kmb_last_error() is set. */
void cuda_block_forward(void *cublas, const float *d_W_in, const float *d_W_out, const float *d_A_log,
                        const float *d_W_B, const float *d_W_C, const float *d_delta_proj, const float *d_theta,
                        const float *d_lambda_proj, const float *d_x, float *d_y, float *d_u_raw, float *d_u,
                        float *d_dt_raw, float *d_dt, float *d_B_exp, float *d_C_exp, float *d_dt_exp,
                        float *d_h_store, float *d_y_scan, float *d_y_proj, float *d_lambda_raw, float *d_lambda,
                        int L, int state, int dim, int R, int spatial_ndims, const long *spatial_dims);
void cuda_block_backward(void *cublas, const float *d_W_in, const float *d_W_out, const float *d_A_log,
                         const float *d_W_B, const float *d_W_C, const float *d_delta_proj, const float *d_theta,
                         const float *d_lambda_proj, const float *d_x, const float *d_u_raw, const float *d_u,
                         const float *d_dt_raw, const float *d_dt, const float *d_B_exp, const float *d_C_exp,
                         const float *d_dt_exp, const float *d_h_store, const float *d_y_scan,
                         const float *d_lambda, const float *d_dy, float *d_dW_in, float *d_dW_out,
                         float *d_dA_log, float *d_dW_B, float *d_dW_C, float *d_ddelta_proj, float *d_g_theta,
                         float *d_g_lambda_proj, float *d_dx, float *d_dy_scan, float *d_du, float *d_du_raw,
                         float *d_ddt, float *d_ddt_raw, float *d_dB_scan, float *d_dC_scan, float *d_ddt_scan,
                         float *d_dA_tmp, float *d_dlambda, float *d_dlambda_raw, int L, int state, int dim, int R,
                         int spatial_ndims, const long *spatial_dims);

#ifdef __cplusplus
}
#endif
#endif
