/* convnd.h -- public C ABI of the B200 dense causal depthwise convND.
 *
 * Struct, enum and entry points follow the reference include/convnd.h:10-99.
 *   out[p,d] = bias[d] + sum_{k in [0,K)^nd} in[p - (K-1-k), d] * kernel[k_lin, d]
 * (zero outside the grid; k_lin row-major over axes, last axis fastest;
 * reference src/convnd.c:396-458).  Backward (src/convnd.c:464-531) zeroes
 * dinput, dkernel and dbias, then writes the full gradients.
 */
#ifndef KMB200_CONVND_H
#define KMB200_CONVND_H

#include "wavefront_plan.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float *input;          /* [P, D] */
    const float *kernel;   /* [K^ndims, D] */
    const float *bias;     /* [D] or NULL */
    float *output;         /* [P, D] */
    float *dy;             /* [P, D] */
    float *dinput;         /* [P, D] */
    float *dkernel;        /* [K^ndims, D] */
    float *dbias;          /* [D] or NULL */
    const long *dims;      /* host memory, [ndims] */
    long ndims;
    long D;
    long K;
} ConvNDParams;

typedef enum {
    CONVND_FORWARD = 1,
    CONVND_BACKWARD = 2,
    CONVND_COMPLETE = 3
} ConvNDMode;

/* reference include/convnd.h:32 */
long convnd_kernel_volume(long ndims, long K);
/* reference include/convnd.h:35,38: run on the GPU after checking the plan. */
void convnd_forward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan);
void convnd_backward_wavefront(ConvNDParams *p, const KMWavefrontPlan *plan);
/* reference include/convnd.h:41 (src/convnd.c:537-573).  Pointers: all device
 * or all host (staged).  void like the reference; the status of the last call
 * on this thread is returned by convnd_status(). */
void convnd(ConvNDParams *p, ConvNDMode mode);
/* reference include/convnd.h:93,96: device pointers, 0 / -1. */
int om_convnd_forward(ConvNDParams *p);
int om_convnd_backward(ConvNDParams *p);

/* ---- additive extensions ---- */
/* 0 if the last convnd()/convnd_*_wavefront() call on this thread succeeded, else -1. */
int convnd_status(void);
/* Batched device-pointer variant: input/output/dy/dinput are [batch, P, D];
 * kernel/bias shared; dkernel/dbias are summed over the batch.  Enqueued on
 * `stream` without synchronising.  mode as ConvNDMode. */
int convnd_batched_async(ConvNDParams *p, long batch, int mode, void *stream);

/* No counterpart in the reference.  The backward of convnd_batched_async
 * (same results up to the order of the dkernel / dbias partial sums, same
 * overwrite semantics, dkernel/dbias summed over the batch) for callers that must not allocate device memory -- e.g. code
 * running under a fixed memory pool or arena, inside allocator hooks, or on
 * paths that may not take the allocator's locks.  It calls no cudaMalloc /
 * cudaFree: its partial sums live in one 4 MiB device array that is part of
 * the loaded library (held on every GPU that loads it until exit), so it
 * rejects (K^ndims + 1) * D > 1048576 with -1.  The first call on a device
 * looks up that array's address; make it before any stream capture, and do
 * not use the entry point across a cudaDeviceReset of that device (the address
 * is kept for the life of the process).  All
 * calls share the array: calls that overlap on the GPU race.  Device
 * pointers only; enqueued on `stream` without synchronising.  0 / -1; the
 * reason of a -1 is returned by convnd_backward_noalloc_error(). */
int convnd_backward_noalloc(ConvNDParams *p, long batch, void *stream);
const char *convnd_backward_noalloc_error(void);

#ifdef __cplusplus
}
#endif
#endif
