/* kmamba_gemm.h -- the matrix products of the block and the LM head
 * (libkmamba_b200.so), exposed for callers that hold their own device buffers.
 * The reference computes these with cuBLAS SGEMM (cuda/mamba_block.cu:357-412,
 * cuda/kmamba_kernels.cu:24-37); here they run on the sm_100a tensor cores.
 *
 * Products (row-major, device pointers, element strides):
 *   trans = 0:  D (+)= A B^T,  A [M, K] (lda), B [N, K] (ldb)
 *   trans = 1:  D (+)= A^T B,  A [K, M] (lda), B [K, N] (ldb)
 * D [M, N] fp32 (ldd); accumulate = 1 adds into D.  0 on success, -1 with
 * kmb_last_error() set otherwise.  Enqueued on `stream` (NULL = default). */
#ifndef KMB200_GEMM_H
#define KMB200_GEMM_H

#ifdef __cplusplus
extern "C" {
#endif

/* How an fp32 product reaches fp32 accuracy. */
#define KMB_GEMM_DEFAULT -1   /* the process-wide kind (kmb_gemm_set_f32_kind) */
#define KMB_GEMM_TF32X3 1     /* 3xTF32: hi/lo tf32 pieces, three tensor-core products */
#define KMB_GEMM_BF16X6 2     /* three bf16 pieces, the six products of order <= 2 */
#define KMB_GEMM_BF16X9 3     /* three bf16 pieces, all nine products */
#define KMB_GEMM_SIMT 4       /* CUDA-core fp32 FMA, fixed K order */

int kmb_gemm_f32(int kind, int trans, long long M, long long N, long long K, const float *A, long long lda,
                 const float *B, long long ldb, float *D, long long ldd, int accumulate, void *stream);
/* bf16 operands, fp32 accumulation and output. */
int kmb_gemm_bf16(int trans, long long M, long long N, long long K, const void *A, long long lda, const void *B,
                  long long ldb, float *D, long long ldd, int accumulate, void *stream);
/* The kind every fp32 product of the block and the model uses. */
int kmb_gemm_set_f32_kind(int kind);
int kmb_gemm_get_f32_kind(void);
/* Tensor-core MMA K steps (16 bf16 / 8 tf32 K each) over which the fp32 kinds let
 * the leading product accumulate in TMEM before the epilogue adds it into an
 * fp32 running sum: 1 .. 64, default 8.  Fewer = closer to an fp32 FMA loop's
 * accuracy, more = fewer TMEM reads.  The smaller products accumulate over all
 * of K and are added once. */
int kmb_gemm_set_f32_flush(int ksteps);
/* Path of this thread's last product: 1 tensor cores, 0 CUDA cores, -1 none yet. */
int kmb_gemm_last_path(void);

#ifdef __cplusplus
}
#endif
#endif
