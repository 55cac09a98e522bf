/* kmamba.h -- k-mamba model API on the B200 (reference include/kmamba.h:238-409).
 *
 * KMambaConfig and MBOptimConfig keep the reference field order and types
 * (include/kmamba.h:238-278, include/kmamba_kernels.h:90-97) so existing
 * config code compiles unchanged.  KMamba is opaque here: every tensor lives
 * in one device arena, every batch item runs through every block at once, and
 * the optimizer is a single multi-tensor AdamW launch over the arena.
 */
#ifndef KMB200_KMAMBA_H
#define KMB200_KMAMBA_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#ifndef KMAMBA_CONFIG_MAX_NDIMS
#define KMAMBA_CONFIG_MAX_NDIMS 32
#endif

typedef struct {
    long max_ndims;
    long max_state;
    int use_fast_exp;
    size_t vocab_size;
    size_t dim;
    size_t state_size;
    size_t seq_len;
    size_t n_layers;
    size_t mimo_rank;
    float dt_scale;
    float dt_min;
    float dt_max;
    float default_lambda;
    int use_a_log_clamp;
    float a_log_min;
    long spatial_ndims;
    long spatial_dims[KMAMBA_CONFIG_MAX_NDIMS];
    int use_convnd;
    int use_convnd_bias;
    long convnd_K;
    long convnd_ndims;
    long pad_left[KMAMBA_CONFIG_MAX_NDIMS];
    long pad_right[KMAMBA_CONFIG_MAX_NDIMS];
    uint32_t d_conv;
    float expand_factor;
    char model_name[64];
    const char **vocab_data;
    int gpu_device;
    int weight_tying;
} KMambaConfig;

typedef struct {
    float lr;
    float mu;            /* AdamW beta1 */
    float beta2;
    float eps;
    float clip_norm;     /* unused by the AdamW step, as in the reference */
    float weight_decay;
} MBOptimConfig;

typedef struct KMamba KMamba;

/* reference src/kmamba.c:308-344 */
void kmamba_config_set_defaults(KMambaConfig *cfg);
void kmamba_optim_config_set_defaults(MBOptimConfig *opt_cfg);
/* reference src/kmamba.c:346-433: validates the config and allocates the
 * device arena on cfg->gpu_device (or the current device). */
KMamba *kmamba_create(const KMambaConfig *cfg);
void kmamba_free(KMamba *m);
/* reference src/kmamba.c:453-466: the reference's own streams, bit for bit:
 * Xavier-uniform embedding (seed) and head (seed + 1), kernels/init_f32.c:38-45;
 * every block from the stream seeded by (dim, state_size, seq_len),
 * src/mamba_block.c:227-268 (A_log = -1, Xavier W_in / W_out / W_B / W_C,
 * theta in [0, 2 pi / N), delta / lambda projections in +-0.01, zero biases;
 * all layers start identical, as in the reference). */
int kmamba_init(KMamba *m, uint32_t seed);
/* The values kmamba_init(seed) gives the tensor `name` ("embedding", "head",
 * "layers.<i>.<field>") of a model with config `cfg`, computed on the host
 * into out[0 .. n) (no device needed).  Returns the element count, or -1 for
 * an unknown name or a short buffer.  No counterpart in the reference. */
long kmb_init_tensor(const KMambaConfig *cfg, uint32_t seed, const char *name, float *out, long n);
/* reference src/kmamba.c:468-486 */
int kmamba_enable_training(KMamba *m, const MBOptimConfig *opt_blocks, float lr_embed_head, float weight_decay);
/* reference src/kmamba.c:626-660: tokens[seq_len] (host) -> logits[seq_len, vocab] (host). */
int kmamba_forward(KMamba *m, const uint32_t *tokens, float *logits_out);
/* reference src/kmamba.c:489-608: batch_tokens[batch, seq_len+1] (host); one
 * forward + backward over the whole batch and one AdamW step.  Returns the mean
 * cross-entropy over batch and positions; the gradient is the exact gradient of
 * that mean (embedding gradient included). */
float kmamba_train_batch(KMamba *m, const uint32_t *batch_tokens, size_t batch_size);
float kmamba_train_step(KMamba *m, const uint32_t *tokens_plus1);
const KMambaConfig *kmamba_get_config(const KMamba *m);
size_t kmamba_step_count(const KMamba *m);
void kmamba_update_lr(KMamba *m, float lr_blocks, float lr_embed);
/* Host copy of a named tensor ("embedding", "head", "layers.<i>.W_in", ...,
 * reference src/kmamba.c:687-738), refreshed by each call; writes to it take
 * effect only through kmamba_set_tensor. */
float *kmamba_get_tensor(KMamba *m, const char *name);
int kmamba_set_tensor(KMamba *m, const char *name, const float *data);

/* ---- extensions (no counterpart in the reference API) ---- */
/* Device-token variants split for data parallelism: forward + backward into
 * the gradient arena (zeroed first); returns the mean loss.  On error it
 * returns NaN and kmb_last_error() is non-empty (a NaN loss with an empty
 * error string is a numerical result: the recurrence overflowed fp32). */
float kmb_model_forward_backward(KMamba *m, const uint32_t *d_batch_tokens, size_t batch_size, void *stream);
/* AdamW over the whole arena (one launch). */
int kmb_model_optimizer_step(KMamba *m, void *stream);
/* Gradient arena (device) and its length in floats, e.g. for an all-reduce. */
float *kmb_model_grad_arena(KMamba *m, size_t *n_floats);
float *kmb_model_param_arena(KMamba *m, size_t *n_floats);
/* Offset and length (floats) of a named tensor inside both arenas. */
int kmb_model_tensor_offset(KMamba *m, const char *name, size_t *offset, size_t *n_floats);

#ifdef __cplusplus
}
#endif
#endif
