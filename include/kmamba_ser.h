/* kmamba_ser.h -- k-mamba models to and from .ser files (reference
 * include/kmamba_ser.h, src/kmamba_ser.c), on libkmamba_b200.so's device
 * model.  Tensor names, order, shapes and the KSerConfig fields are the
 * reference's.  Differences, each a fix:
 *   - every layers.<i>.<field> tensor is saved and loaded under its own name
 *     (the reference's kmamba_get_tensor / kmamba_set_tensor resolve all of them
 *     to W_in, src/kmamba.c:687-738, so its files carry W_in in every slot);
 *   - the loader takes mimo_rank from the W_in shape (KSerConfig has no field
 *     for it; the reference's loader leaves it at 1);
 *   - KM_SER_VERIFY works (the reference never computes the checksum on POSIX). */
#ifndef KMB200_KMAMBA_SER_H
#define KMB200_KMAMBA_SER_H

#include "kmamba.h"
#include "kser.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KM_SER_LAZY 0x01
#define KM_SER_VERIFY 0x02

typedef struct {
    KSerInfo base;
    uint32_t n_layers;
    uint32_t state_size;
    uint32_t seq_len;
} KMSerInfo;

/* reference src/kmamba_ser.c:16-166: embedding, then per layer W_in, W_out,
 * A_log, W_B, W_C, delta_proj, lambda_proj, b_B, b_C, theta, then head, each
 * stored as `dtype`.  KSER_OK or a KSerError. */
int kmamba_save_ser(KMamba *m, const char *path, KSerDtype dtype);
/* reference src/kmamba_ser.c:176-241: a new model (kmamba_config_set_defaults
 * + the file's config) on the current device, every tensor loaded.  NULL on
 * failure (message in kmb_last_error()). */
KMamba *kmamba_load_ser(const char *path, int flags);
/* kmamba_load_ser with the caller's config for the fields a .ser file does not
 * carry (spatial_ndims / spatial_dims, dt_*, lambda, gpu_device): the file's
 * vocab_size, dim, state_size, n_layers, seq_len, d_conv, expand_factor and
 * model_name override `base`.  No counterpart in the reference. */
KMamba *kmb_load_ser_ex(const char *path, int flags, const KMambaConfig *base);
/* reference src/kmamba_ser.c:246-259 (state_size and seq_len filled here). */
KMSerInfo kmamba_ser_info(const char *path);
/* reference src/kmamba_ser.c:264-284: weights only, as the reference. */
int kmamba_save_checkpoint_ser(KMamba *m, void *opt, const char *path, KSerDtype dtype);
int kmamba_load_checkpoint_ser(const char *path, KMamba **m_out, void **opt_out, int flags);

#ifdef __cplusplus
}
#endif
#endif
