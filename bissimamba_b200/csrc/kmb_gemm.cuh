// kmb_gemm.cuh -- the tensor-core GEMM (gemm_tc.cu) and its helpers, shared by
// the block and model products (block_gemm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kmb {

// One GEMM operand: up to three pieces with a common row stride (elements).
// K-major: rows x K row-major; MN-major: K x rows row-major.
struct GemmOperand {
    const void* p[3];
    long long ld;
    int mn_major;
};

// D[m, n] (+)= sum_k A[m, k] B[n, k] on the tensor cores.  kind: 0 bf16, 1 3xTF32
// (pieces hi, lo), 2 / 3 split-bf16 with 6 / 9 products (pieces b0, b1, b2).
// epi: 0 store, 1 add.  cudaErrorNotSupported when the shapes or alignments do
// not fit.
cudaError_t gemm_tc(int kind, int epi, long long M, long long N, long long K, const GemmOperand& A,
                    const GemmOperand& B, float* D, long long ldd, int nsplit, long long split_stride, int* status,
                    cudaStream_t st);
cudaError_t gemm_split(int kind, const float* x, void* const* out, long long rows, long long cols, long long ldx,
                       long long ldo, cudaStream_t st);
cudaError_t gemm_transpose_f32(const float* in, float* out, long long R, long long Cn, long long ldi, long long ldo,
                               cudaStream_t st);
cudaError_t gemm_transpose_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, long long R, long long Cn,
                                long long ldi, long long ldo, cudaStream_t st);
cudaError_t gemm_reduce_splits(const float* part, float* out, long long rows, long long cols, int nsplit,
                               long long split_stride, long long ldp, long long ldo, int accumulate, cudaStream_t st);

}  // namespace kmb
