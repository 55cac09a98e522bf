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
/* 1 = route every forward through the generic kernel (tests / comparison). */
void kmb_set_force_generic(int on);
#ifdef __cplusplus
}
#endif
#endif
