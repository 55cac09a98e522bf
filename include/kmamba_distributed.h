/* kmamba_distributed.h -- one process per GPU over NCCL (NVLink / NVSwitch on
 * one node): the rebuild of the reference's include/kmamba_distributed.h and
 * cuda/kmamba_distributed.cu, whose NCCL path never exchanged the unique id
 * (cuda/kmamba_distributed.cu:46-50) and was never called.
 *
 * The scans and convnd shard by batch item with no exchange in the forward;
 * the collectives are the final output gather (forward), the all-reduce of the
 * weight gradients (backward: dA / dtheta of Scan-A, dkernel / dbias of
 * convnd, the model's gradient arena) and the parameter broadcast. */
#ifndef KMB200_DISTRIBUTED_H
#define KMB200_DISTRIBUTED_H

#include <stddef.h>
#include <stdint.h>

#include "convnd.h"
#include "kmamba.h"
#include "scan_nd.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference include/kmamba_distributed.h:17-33 (same fields, same order) */
typedef struct {
    int world_size;
    int rank;
    int local_rank;
    size_t layer_start, layer_end;
    size_t batch_start, batch_end;
    int use_nccl;
    int use_p2p;
} KMambaDistributedConfig;

/* Opaque NCCL context (the reference exposes its struct; here it is opaque). */
typedef struct KMambaDistributedContext KMambaDistributedContext;

/* reference src/kmamba_distributed.c:120-139: [batch_start, batch_end) of
 * cfg->rank; earlier ranks take the extra items. */
void kmamba_distributed_split_batch(KMambaDistributedConfig *cfg, size_t batch_size, size_t total_gpus);
/* reference src/kmamba_distributed.c:141-160: the same rule over layers. */
void kmamba_distributed_split_layers(KMambaDistributedConfig *cfg, size_t n_layers, size_t total_gpus);

/* reference cuda/kmamba_distributed.cu:22-69.  world_size ranks, this one
 * `rank`, on device LOCAL_RANK (environment) or `rank`.  Rank 0 creates the
 * NCCL unique id and sends it to the others over TCP: it listens on
 * MASTER_ADDR (default 127.0.0.1), port KMB_NCCL_PORT (default MASTER_PORT + 1);
 * the others connect, retrying for up to 120 s.  NULL on failure (message in
 * kmb_last_error()).  world_size 1 gives a context whose collectives are
 * no-ops. */
KMambaDistributedContext *kmamba_distributed_init_nccl(int world_size, int rank);
/* reference cuda/kmamba_distributed.cu:71-84 */
void kmamba_distributed_fini_nccl(KMambaDistributedContext *ctx);
/* reference cuda/kmamba_distributed.cu:86-110: in-place sum over the ranks,
 * synchronous.  0 / -1. */
int kmamba_allreduce_gradients_nccl(KMambaDistributedContext *ctx, float *d_gradients, size_t n_elements);
/* reference cuda/kmamba_distributed.cu:112-138: rank 0's values to every rank, synchronous. */
int kmamba_broadcast_params_nccl(KMambaDistributedContext *ctx, float *d_params, size_t n_elements);

/* ---- additive (no counterpart in the reference) ---- */
/* The 128-byte NCCL unique id (rank 0 creates it; the caller distributes it
 * by any means, e.g. its own launcher's store). */
int kmb_dist_unique_id(void *id128);
/* Context from an id the caller already distributed; device < 0 = current. */
KMambaDistributedContext *kmb_dist_init(const void *id128, int world_size, int rank, int device);
/* The TCP id exchange used by kmamba_distributed_init_nccl (no GPU needed):
 * rank 0 sends id128 to the other world_size - 1 ranks, which receive it into
 * id128.  addr / port as above when NULL / 0.  0 / -1. */
int kmb_dist_exchange_id(void *id128, int world_size, int rank, const char *addr, int port);
int kmb_dist_world_size(const KMambaDistributedContext *ctx);
int kmb_dist_rank(const KMambaDistributedContext *ctx);
/* Asynchronous collectives on `stream` (NULL = the context's own stream).
 * allreduce: buf <- scale * sum over ranks (scale applied after the sum).
 * allgather: recv[r * count .. (r + 1) * count) <- rank r's send[0 .. count);
 * every rank must pass the same count (pad uneven shards), as NCCL requires;
 * with KMB_DIST_CHECK set in the environment the counts are compared first and
 * a mismatch returns -1 instead of hanging. */
int kmb_dist_allreduce_async(KMambaDistributedContext *ctx, float *buf, size_t count, float scale, void *stream);
int kmb_dist_allgather_async(KMambaDistributedContext *ctx, const float *send, float *recv, size_t count,
                             void *stream);
int kmb_dist_broadcast_async(KMambaDistributedContext *ctx, float *buf, size_t count, int root, void *stream);
/* Batch-sharded Scan-A backward: this rank's items as scannd_backward_ex
 * (per-item gradients dB, dC, ddelta, dlambda, dx are local), then dA and
 * dtheta hold the sum over every rank's items: added to (overwrite = 0) or
 * assigned to (overwrite = 1) the caller's buffers, identical on all ranks. */
int kmb_dist_scannd_backward(KMambaDistributedContext *ctx, ScanNDParams *p, long local_batch, float *dx,
                             int overwrite, void *stream);
/* Batch-sharded convnd backward (convnd_batched_async, mode BACKWARD): dinput
 * local; dkernel / dbias the sum over every rank's items on all ranks. */
int kmb_dist_convnd_backward(KMambaDistributedContext *ctx, ConvNDParams *p, long local_batch, void *stream);
/* Data-parallel model step: this rank's sequences d_tokens[local_batch,
 * seq_len + 1] (device), gradient arena scaled by local_batch / global_batch
 * and summed over the ranks (so it is the gradient of the global mean loss),
 * then one AdamW step on every rank.  Returns the global mean loss (NaN on
 * error). */
float kmb_dist_model_train_step(KMambaDistributedContext *ctx, KMamba *m, const uint32_t *d_tokens,
                                size_t local_batch, size_t global_batch, void *stream);

#ifdef __cplusplus
}
#endif
#endif
