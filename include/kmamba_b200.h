/* kmamba_b200.h -- diagnostics of libkmamba_b200.so (no counterpart in the
 * reference API; the reference reports errors only through return codes). */
#ifndef KMB200_DIAG_H
#define KMB200_DIAG_H
#ifdef __cplusplus
extern "C" {
#endif
/* Text of the last error raised on this host thread ("" if none). */
const char *kmb_last_error(void);
/* Empty the last-error text of this host thread. */
void kmb_clear_error(void);
/* Synchronise `stream` and return the device status word of this host thread
 * and device, then clear it: 0 = no kernel gave up waiting, > 0 = the code of
 * the first bounded wait that ran out (asynchronous entry points record it
 * there instead of failing), -1 = CUDA error. */
int kmb_device_status(void *stream);
/* Which Scan-A forward kernel the last forward call on this thread used:
 * 1 = persistent TMA kernel (1D/2D fast path), 0 = generic kernel, -1 = none. */
int kmb_last_forward_path(void);
/* Which Scan-A backward kernel the last backward call on this thread used:
 * 2 = 2D systolic strips, 1 = level-parallel wave kernel, 0 = generic. */
int kmb_last_backward_path(void);
/* 1 = route every forward through the generic kernel (tests / comparison). */
void kmb_set_force_generic(int on);
/* Exponential of the 2D Scan-A forward (process-wide).  0 (default): expf of
 * delta*A with the reference's operation order (src/scan_nd.c:126-168), within
 * 1e-4 rel / 1e-5 abs of the reference's fp32 result.  1 (opt-in, faster):
 * one ex2.approx of delta*(A log2 e) and a re-associated trapezoid term; it is
 * a few ulp per update from expf, which the recurrence compounds. */
void kmb_set_scan_exp2(int on);
/* Persistent kernels (the Scan-A strip and TMA kernels) size their grid to the
 * SM count minus n (process-wide, default 0), so that a communication kernel
 * enqueued on another stream (an NCCL gather overlapping the scan) finds SMs
 * free instead of waiting for the scan to end. */
void kmb_set_sm_reserve(int n);
int kmb_get_scan_exp2(void);
#ifdef __cplusplus
}
#endif
#endif
