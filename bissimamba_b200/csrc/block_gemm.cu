// block_gemm.cu -- the block's and the LM head's matrix products without a
// library: the large ones on the tensor cores (gemm_tc.cu: bf16, or fp32 at
// fp32 accuracy from split-bf16 or 3xTF32 pieces), the rank-R ones (K or N =
// R, the MIMO rank) and the column sums as memory-bound kernels of their own,
// every reduction in a fixed order.
//
// Front-ends (all enqueue on `st`):
//   mm_nt   D (+)= A B^T with A [M, K], B [N, K] row-major (K-major operands);
//   mm_tn   D (+)= A^T B with A [K, M], B [K, N] row-major: MN-major operands
//           (bf16 and the split-bf16 pieces read in place; 3xTF32 transposes
//           first), K (the long batch-row axis) split over CTAs, the partials
//           added in split order;
//   rank_rows    out[row, r]  = sum_j X[row, j] W[j, r]      (dy = dout W_out)
//   rank_outer   G[j, r]     += sum_row X[row, j] Y[row, r]  (dW_out += dout^T y)
//   col_sums     g[j]        += sum_row X[row, j]            (bias gradients)
//   out_rank     out[row, j]  = x[row, j] + sum_r y[row, r] W[j, r]
// A SIMT tile kernel takes the shapes the tensor-core kernel does not (unaligned
// strides), so no path falls back to a library GEMM.
#include <cuda_bf16.h>
#include "kmb_common.cuh"
#include "kmb_gemm.cuh"

namespace kmb {

void* workspace(int slot, size_t bytes);
int* device_status();
int set_error(const char* msg);
int set_cuda_error(const char* where, cudaError_t e);
void clear_error();
int gemm_set_kflush(int k);
enum { KIND_BF16_ = 0, KIND_TF32X3_ = 1, KIND_BF16X6_ = 2, KIND_BF16X9_ = 3, KIND_SIMT_ = 4 };
enum { WS_GEMM_A = 12, WS_GEMM_B = 13, WS_GEMM_T = 15, WS_GEMM_P = 16 };   // workspace slots

// kind of the fp32 products (process-wide; kmb_gemm_set_f32_kind)
static int g_f32_kind = KIND_BF16X6_;
static thread_local int tl_gemm_path = -1;   // last product: 1 tensor cores, 0 SIMT

namespace {

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// D[m, n] (+)= sum_k A[m, k] B[n, k]: 32 x 32 output tile per block, fixed k order
template <typename T>
__global__ void gemm_simt_nt(long long M, long long N, long long K, const T* __restrict__ A, long long lda,
                             const T* __restrict__ B, long long ldb, float* __restrict__ D, long long ldd, int acc) {
    __shared__ float sa[32][33], sb[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 256 threads: 32 x 8
    const long long m0 = (long long)blockIdx.y * 32, n0 = (long long)blockIdx.x * 32;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    for (long long k0 = 0; k0 < K; k0 += 32) {
        for (int i = ty; i < 32; i += 8) {
            const long long m = m0 + i, n = n0 + i, k = k0 + tx;
            sa[i][tx] = (m < M && k < K) ? ldf(A + m * lda + k) : 0.0f;
            sb[i][tx] = (n < N && k < K) ? ldf(B + n * ldb + k) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; k++) {
            const float bv = sb[tx][k];
#pragma unroll
            for (int j = 0; j < 4; j++) c[j] = __fmaf_rn(sa[ty + 8 * j][k], bv, c[j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const long long m = m0 + ty + 8 * j, n = n0 + tx;
        if (m < M && n < N) {
            float* o = D + m * ldd + n;
            *o = acc ? *o + c[j] : c[j];
        }
    }
}

// out[row, r] = sum_j X[row, j] W[j, r] for r in [r0, r0 + 4) and < R: one warp
// per row, lanes stride the row, a butterfly adds the lanes (fixed order)
template <typename T>
__global__ void rank_rows_kernel(const T* __restrict__ X, const float* __restrict__ W, long long rows, int dim, int R,
                                 int r0, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const T* x = X + row * dim;
    for (int j = lane; j < dim; j += 32) {
        const float v = ldf(x + j);
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (r0 + r < R) acc[r] = __fmaf_rn(v, W[(long long)j * R + r0 + r], acc[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(~0u, acc[r], o);
    if (lane < 4 && r0 + lane < R)
        out[row * R + r0 + lane] = lane == 0 ? acc[0] : lane == 1 ? acc[1] : lane == 2 ? acc[2] : acc[3];
}

// part[chunk][j][r] = sum over the chunk's rows of X[row, j] Y[row, r] for r in
// [r0, r0 + 4) and < R (Y == nullptr: Y = 1, r = 0)
template <typename T>
__global__ void outer_partials(const T* __restrict__ X, const float* __restrict__ Y, long long rows, int dim, int R,
                               int r0, long long rows_per_chunk, float* __restrict__ part) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= dim) return;
    const long long q0 = (long long)blockIdx.y * rows_per_chunk, q1 = min(rows, q0 + rows_per_chunk);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (long long row = q0; row < q1; row++) {
        const float v = ldf(X + row * dim + j);
        if (!Y) {
            acc[0] += v;
        } else {
#pragma unroll
            for (int r = 0; r < 4; r++)
                if (r0 + r < R) acc[r] = __fmaf_rn(v, Y[row * R + r0 + r], acc[r]);
        }
    }
    const int RR = Y ? R : 1;
#pragma unroll
    for (int r = 0; r < 4; r++)
        if (r0 + r < RR) part[((long long)blockIdx.y * dim + j) * RR + r0 + r] = acc[r];
}

// out[i] += sum_c part[c][i], fixed order
__global__ void add_partials(const float* __restrict__ part, long long n, int nchunk, float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float acc = 0.0f;
    for (int c = 0; c < nchunk; c++) acc += part[(long long)c * n + i];
    out[i] += acc;
}

// The rank-R products of the block backward in one pass over X [rows, dim]
// (dout, or dB / dC for the bias sums), for ranks r0 .. r0 + rc - 1 (rc <= RM):
//   dy[row, r]           = sum_j X[row, j] W[j, r]              (dy non-null)
//   part[blk][j][r - r0] = sum over the block's rows of X[row, j] Y[row, r]
//                          (part non-null; Y == nullptr: Y = 1, rc = 1)
// One warp per row; lane l holds NC chunks of V consecutive columns (16-byte
// loads) at (c * 32 + l) * V, and the next row's chunks are loaded before the
// current row is used.  dy is a butterfly over the lanes; the block's eight
// warps add their column partials into shared memory in warp order.  Every
// sum has a fixed order.
template <typename T, int NC, int RM>
__global__ void __launch_bounds__(256, (NC * (16 / (int)sizeof(T)) * RM <= 16 || (sizeof(T) == 2 && NC <= 2 && NC * RM <= 4)) ? 2 : 1)
rank_pass(const T* __restrict__ X, const float* __restrict__ W, const float* __restrict__ Y, long long rows, int dim,
          int R, int r0, int rc, float* __restrict__ dy, float* __restrict__ part) {
    constexpr int V = 16 / sizeof(T);
    extern __shared__ float rp_buf[];   // [dim][RM]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float acc[NC][V][RM];
    float wv[NC][V][RM];
#pragma unroll
    for (int c = 0; c < NC; c++)
#pragma unroll
        for (int v = 0; v < V; v++)
#pragma unroll
            for (int r = 0; r < RM; r++) {
                acc[c][v][r] = 0.0f;
                const int j = (c * 32 + lane) * V + v;
                wv[c][v][r] = (dy && j < dim && r < rc) ? W[(long long)j * R + r0 + r] : 0.0f;
            }
    const long long stride = (long long)gridDim.x * 8;
    long long row = (long long)blockIdx.x * 8 + warp;
    // two rows in flight ahead of the one in use: X chunks and the row's Y values
    uint4 b0[NC], b1[NC];
    float y0[RM], y1[RM];
    auto load = [&](uint4 (&dst)[NC], float (&yd)[RM], long long rw) {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int j0 = (c * 32 + lane) * V;
            dst[c] = (rw < rows && j0 < dim) ? __ldcs(reinterpret_cast<const uint4*>(X + rw * dim + j0))
                                             : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int r = 0; r < RM; r++)
            yd[r] = Y ? ((r < rc && rw < rows) ? Y[rw * R + r0 + r] : 0.0f) : (r == 0 ? 1.0f : 0.0f);
    };
    load(b0, y0, row);
    load(b1, y1, row + stride);
    for (; row < rows; row += stride) {
        float xv[NC][V];
        float yr[RM];
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const T* e = reinterpret_cast<const T*>(&b0[c]);
#pragma unroll
            for (int v = 0; v < V; v++) xv[c][v] = ldf(e + v);
            b0[c] = b1[c];
        }
#pragma unroll
        for (int r = 0; r < RM; r++) {
            yr[r] = y0[r];
            y0[r] = y1[r];
        }
        load(b1, y1, row + 2 * stride);
        if (part) {
#pragma unroll
            for (int c = 0; c < NC; c++)
#pragma unroll
                for (int v = 0; v < V; v++)
#pragma unroll
                    for (int r = 0; r < RM; r++) acc[c][v][r] = __fmaf_rn(xv[c][v], yr[r], acc[c][v][r]);
        }
        if (dy) {
            float sr[RM];
#pragma unroll
            for (int r = 0; r < RM; r++) sr[r] = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; c++)
#pragma unroll
                for (int v = 0; v < V; v++)
#pragma unroll
                    for (int r = 0; r < RM; r++) sr[r] = __fmaf_rn(xv[c][v], wv[c][v][r], sr[r]);
#pragma unroll
            for (int r = 0; r < RM; r++)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sr[r] += __shfl_xor_sync(~0u, sr[r], o);
#pragma unroll
            for (int r = 0; r < RM; r++)
                if (lane == r && r < rc) dy[row * R + r0 + r] = sr[r];
        }
    }
    if (!part) return;
    // block partial: warps add in order 0..7
    for (int w = 0; w < 8; w++) {
        if (warp == w) {
#pragma unroll
            for (int c = 0; c < NC; c++)
#pragma unroll
                for (int v = 0; v < V; v++) {
                    const int j = (c * 32 + lane) * V + v;
                    if (j < dim)
#pragma unroll
                        for (int r = 0; r < RM; r++) {
                            float* b = rp_buf + j * RM + r;
                            *b = w == 0 ? acc[c][v][r] : *b + acc[c][v][r];
                        }
                }
        }
        __syncthreads();
    }
    const int rr = Y ? rc : 1;
    float* out = part + (long long)blockIdx.x * dim * rr;   // [dim][rr]
    for (int i = threadIdx.x; i < dim * rr; i += blockDim.x) out[i] = rp_buf[(i / rr) * RM + (i % rr)];
}

// G[j, r0 + r] += sum_b part[b][j][r]: 32 elements per block, warp w adds the blocks w, w + 8, ...
// in order, then warp 0 adds the eight warp sums in order (a fixed order overall)
__global__ void add_rank_partials(const float* __restrict__ part, int nblk, int dim, int rr, int R, int r0,
                                  float* __restrict__ G) {
    __shared__ float ws[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * 32 + lane;
    const int n = dim * rr;
    float acc = 0.0f;
    if (i < n) {
        // blocks warp, warp + 8, ... added in that order; eight loads issued before their adds
        int b = warp;
        for (; b + 56 < nblk; b += 64) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; k++) v[k] = part[(long long)(b + 8 * k) * n + i];
#pragma unroll
            for (int k = 0; k < 8; k++) acc += v[k];
        }
        for (; b < nblk; b += 8) acc += part[(long long)b * n + i];
    }
    ws[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && i < n) {
        float t = ws[0][lane];
#pragma unroll
        for (int w = 1; w < 8; w++) t += ws[w][lane];
        const int j = i / rr, r = i - j * rr;
        G[(long long)j * R + r0 + r] += t;
    }
}

// out[row, j] = x[row, j] + sum_r y[row, r] W[j, r], four columns per thread (dim % 4 == 0).
// W (dim x R) is staged once per CTA in shared memory as its transpose [R][dim], so a thread reads its four
// columns of each rank as one conflict-free 16-byte load (read from W directly, the R x 4 scalars of a
// thread sit 16 R bytes apart across the warp and each load touched ~16 sectors).  A CTA walks rows
// (rpi rows at a time, tpr threads per row, grid-stride); the sum over r is in ascending order.
__global__ void out_rank_f32x4(const float4* __restrict__ x, const float* __restrict__ y, const float* __restrict__ W,
                               long long rows, int dim4, int R, float4* __restrict__ out) {
    extern __shared__ float4 ork_wt[];   // [R][dim4]
    const int dim = dim4 * 4;
    float* wt = (float*)ork_wt;
    for (int i = threadIdx.x; i < dim * R; i += blockDim.x) {
        const int j = i / R, r = i - j * R;
        wt[r * dim + j] = W[i];
    }
    __syncthreads();
    const int tpr = dim4 < (int)blockDim.x ? dim4 : (int)blockDim.x;
    const int rpi = blockDim.x / tpr;
    const int sub = threadIdx.x / tpr, c0 = threadIdx.x - sub * tpr;
    if (sub >= rpi) return;
    // four rows per step (their loads in flight together)
    const long long rstep = (long long)gridDim.x * rpi;
    for (long long row0 = (long long)blockIdx.x * rpi + sub; row0 < rows; row0 += 4 * rstep) {
        for (int j4 = c0; j4 < dim4; j4 += tpr) {
            float4 xv[4], a[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const long long row = row0 + q * rstep;
                a[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row < rows) xv[q] = x[row * dim4 + j4];
            }
            for (int r = 0; r < R; r++) {
                const float4 w = ork_wt[r * dim4 + j4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const long long row = row0 + q * rstep;
                    const float yv = row < rows ? y[row * R + r] : 0.0f;
                    a[q].x = __fmaf_rn(yv, w.x, a[q].x);
                    a[q].y = __fmaf_rn(yv, w.y, a[q].y);
                    a[q].z = __fmaf_rn(yv, w.z, a[q].z);
                    a[q].w = __fmaf_rn(yv, w.w, a[q].w);
                }
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const long long row = row0 + q * rstep;
                if (row < rows)
                    out[row * dim4 + j4] = make_float4(xv[q].x + a[q].x, xv[q].y + a[q].y, xv[q].z + a[q].z,
                                                       xv[q].w + a[q].w);
            }
        }
    }
}

// out[row, j] = x[row, j] + sum_r y[row, r] W[j, r]   (fp32 residual stream)
__global__ void out_rank_f32(const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ W,
                             long long rows, int dim, int R, float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * dim) return;
    const long long row = i / dim;
    const int j = (int)(i - row * dim);
    float acc = 0.0f;
    for (int r = 0; r < R; r++) acc = __fmaf_rn(y[row * R + r], W[(long long)j * R + r], acc);
    out[i] = x[i] + acc;
}

unsigned nblk(long long n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

cudaError_t rank_bwd(bool bf16, const void* X, const float* W, const float* Y, long long rows, int dim, int R,
                     float* dy, float* G, cudaStream_t st);

static int npieces(int kind) { return kind == KIND_BF16_ ? 1 : kind == KIND_TF32X3_ ? 2 : 3; }

// What the last split of this host thread left in the A / B piece workspaces
struct PieceKey {
    const float* x;
    long long rows, cols, ldx, ldo;
    int kind;
    const void* buf;
};
static thread_local PieceKey tl_pieces[2];

// The pieces of the fp32 matrix x [rows, cols] (stride ldx) in workspace `slot`, row stride ldo
// (a multiple of 8 elements, so rows are 16-byte aligned for either element size).  With `unchanged`
// (the caller guarantees x was not written since this thread's previous split of it), pieces still in
// the workspace from a split of the same matrix in the same layout are used as they are.
static cudaError_t make_pieces(int kind, int slot, const float* x, long long rows, long long cols, long long ldx,
                               long long ldo, GemmOperand& op, cudaStream_t st, bool unchanged = false) {
    const int np = npieces(kind);
    const size_t esz = kind == KIND_TF32X3_ ? 4 : 2;
    const size_t one = ((size_t)rows * ldo * esz + 255) & ~(size_t)255;
    char* w = (char*)workspace(slot, one * np);
    if (!w) return cudaErrorMemoryAllocation;
    void* out[3] = {w, np > 1 ? w + one : nullptr, np > 2 ? w + 2 * one : nullptr};
    for (int p = 0; p < 3; p++) op.p[p] = out[p];
    op.ld = ldo;
    PieceKey& key = tl_pieces[slot == WS_GEMM_A ? 0 : 1];
    const PieceKey now{x, rows, cols, ldx, ldo, kind, w};
    if (unchanged && key.x == now.x && key.rows == rows && key.cols == cols && key.ldx == ldx && key.ldo == ldo &&
        key.kind == kind && key.buf == w)
        return cudaSuccess;
    key = PieceKey{};
    const cudaError_t e = gemm_split(kind, x, out, rows, cols, ldx, ldo, st);
    if (e == cudaSuccess) key = now;
    return e;
}

static cudaError_t simt_nt(bool bf16, long long M, long long N, long long K, const void* A, long long lda,
                           const void* B, long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st) {
    dim3 grid(nblk(N, 32), nblk(M, 32));
    if (bf16)
        gemm_simt_nt<__nv_bfloat16><<<grid, 256, 0, st>>>(M, N, K, (const __nv_bfloat16*)A, lda,
                                                          (const __nv_bfloat16*)B, ldb, D, ldd, accumulate);
    else
        gemm_simt_nt<float><<<grid, 256, 0, st>>>(M, N, K, (const float*)A, lda, (const float*)B, ldb, D, ldd,
                                                  accumulate);
    tl_gemm_path = 0;
    return cudaGetLastError();
}

static inline long long round8(long long v) { return (v + 7) & ~7LL; }

// D (+)= A B^T: bf16 inputs, or fp32 inputs at fp32 accuracy (kind: the fp32 kind, or
// KIND_SIMT_ for the CUDA-core kernel).  A [M, K] (lda), B [N, K] (ldb).
static cudaError_t mm_nt_kind(int kind, bool bf16, long long M, long long N, long long K, const void* A,
                              long long lda, const void* B, long long ldb, float* D, long long ldd, bool accumulate,
                              cudaStream_t st, bool a_unchanged = false) {
    int* status = device_status();
    cudaError_t e = cudaErrorNotSupported;
    if (status && (bf16 || kind != KIND_SIMT_)) {
        if (bf16) {
            const GemmOperand a{{A, nullptr, nullptr}, lda, 0}, b{{B, nullptr, nullptr}, ldb, 0};
            e = gemm_tc(KIND_BF16_, accumulate ? 1 : 0, M, N, K, a, b, D, ldd, 1, 0, status, st);
        } else {
            GemmOperand a{}, b{};
            const long long ldk = round8(K);
            if ((e = make_pieces(kind, WS_GEMM_A, (const float*)A, M, K, lda, ldk, a, st, a_unchanged)) != cudaSuccess)
                return e;
            if ((e = make_pieces(kind, WS_GEMM_B, (const float*)B, N, K, ldb, ldk, b, st)) != cudaSuccess) return e;
            e = gemm_tc(kind, accumulate ? 1 : 0, M, N, K, a, b, D, ldd, 1, 0, status, st);
        }
        if (e == cudaSuccess) tl_gemm_path = 1;
    }
    if (e != cudaErrorNotSupported) return e;
    cudaGetLastError();
    return simt_nt(bf16, M, N, K, A, lda, B, ldb, D, ldd, accumulate, st);
}

cudaError_t mm_nt(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st) {
    return mm_nt_kind(g_f32_kind, bf16, M, N, K, A, lda, B, ldb, D, ldd, accumulate, st);
}

// mm_nt whose A the previous product of this thread split in the same layout (an mm_tn's A [K, M] split
// rows = K is the same matrix as an mm_nt's A [M, K]) and nothing wrote since: its pieces are reused.
cudaError_t mm_nt_same_a(bool bf16, long long M, long long N, long long K, const void* A, long long lda,
                         const void* B, long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st) {
    return mm_nt_kind(g_f32_kind, bf16, M, N, K, A, lda, B, ldb, D, ldd, accumulate, st, true);
}

// D[M, N] (+)= A^T B with A [K, M] (lda), B [K, N] (ldb).  K is split over
// CTAs so that the output tiles fill the SMs; the partials are summed in
// split order.
static cudaError_t mm_tn_kind(int kind, bool bf16, long long M, long long N, long long K, const void* A,
                              long long lda, const void* B, long long ldb, float* D, long long ldd, bool accumulate,
                              cudaStream_t st) {
    const bool pieces_mn = !bf16 && (kind == KIND_BF16X6_ || kind == KIND_BF16X9_);
    const bool direct = bf16 || pieces_mn;   // MN-major operands read in place
    const long long tiles = ((M + 127) / 128) * ((N + (bf16 ? 255 : 191)) / (bf16 ? 256 : 192));
    int nsplit = (int)((148 + tiles - 1) / tiles);
    const long long kb = (K + 63) / 64;
    if (nsplit > kb) nsplit = (int)kb;
    if (nsplit < 1) nsplit = 1;
    float* part = (float*)workspace(WS_GEMM_P, (size_t)nsplit * M * N * sizeof(float));
    int* status = device_status();
    if (!part || !status) return cudaErrorMemoryAllocation;
    cudaError_t e = cudaErrorNotSupported;
    if (direct && (bf16 || kind != KIND_SIMT_)) {
        GemmOperand a{}, b{};
        if (bf16) {
            a = GemmOperand{{A, nullptr, nullptr}, lda, 1};
            b = GemmOperand{{B, nullptr, nullptr}, ldb, 1};
        } else {
            if ((e = make_pieces(kind, WS_GEMM_A, (const float*)A, K, M, lda, round8(M), a, st)) != cudaSuccess)
                return e;
            if ((e = make_pieces(kind, WS_GEMM_B, (const float*)B, K, N, ldb, round8(N), b, st)) != cudaSuccess)
                return e;
            a.mn_major = b.mn_major = 1;
        }
        e = gemm_tc(bf16 ? KIND_BF16_ : kind, 0, M, N, K, a, b, part, N, nsplit, M * N, status, st);
        if (e == cudaErrorNotSupported) cudaGetLastError();
    }
    if (e == cudaErrorNotSupported) {
        // transpose into K-major scratch ([M, K] and [N, K], K padded to a multiple of 8), then nt
        const long long Kp = round8(K);
        const size_t esz = bf16 ? 2 : 4;
        char* ta = (char*)workspace(WS_GEMM_T, (size_t)(M + N) * Kp * esz + 512);
        if (!ta) return cudaErrorMemoryAllocation;
        char* tb = ta + (((size_t)M * Kp * esz + 255) & ~(size_t)255);
        if (bf16) {
            if ((e = gemm_transpose_bf16((const __nv_bfloat16*)A, (__nv_bfloat16*)ta, K, M, lda, Kp, st)) !=
                    cudaSuccess ||
                (e = gemm_transpose_bf16((const __nv_bfloat16*)B, (__nv_bfloat16*)tb, K, N, ldb, Kp, st)) !=
                    cudaSuccess)
                return e;
        } else {
            if ((e = gemm_transpose_f32((const float*)A, (float*)ta, K, M, lda, Kp, st)) != cudaSuccess ||
                (e = gemm_transpose_f32((const float*)B, (float*)tb, K, N, ldb, Kp, st)) != cudaSuccess)
                return e;
        }
        e = cudaErrorNotSupported;
        if (bf16 || kind != KIND_SIMT_) {
            GemmOperand a{}, b{};
            if (bf16) {
                a = GemmOperand{{ta, nullptr, nullptr}, Kp, 0};
                b = GemmOperand{{tb, nullptr, nullptr}, Kp, 0};
            } else {
                if ((e = make_pieces(kind, WS_GEMM_A, (const float*)ta, M, K, Kp, Kp, a, st)) != cudaSuccess) return e;
                if ((e = make_pieces(kind, WS_GEMM_B, (const float*)tb, N, K, Kp, Kp, b, st)) != cudaSuccess) return e;
            }
            e = gemm_tc(bf16 ? KIND_BF16_ : kind, 0, M, N, K, a, b, part, N, nsplit, M * N, status, st);
        }
        if (e == cudaErrorNotSupported) {
            cudaGetLastError();
            nsplit = 1;
            e = simt_nt(bf16, M, N, K, ta, Kp, tb, Kp, part, N, false, st);
        } else if (e == cudaSuccess) {
            tl_gemm_path = 1;
        }
    } else if (e == cudaSuccess) {
        tl_gemm_path = 1;
    }
    if (e != cudaSuccess) return e;
    return gemm_reduce_splits(part, D, M, N, nsplit, M * N, N, ldd, accumulate ? 1 : 0, st);
}

cudaError_t mm_tn(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st) {
    return mm_tn_kind(g_f32_kind, bf16, M, N, K, A, lda, B, ldb, D, ldd, accumulate, st);
}

// One pass of rank_pass per group of four ranks: dy (if non-null) and G += X^T Y (if G non-null; Y ==
// nullptr: G[j] += column sums).  cudaErrorNotSupported when the row layout does not fit the kernel.
static cudaError_t rank_pass_run(bool bf16, const void* X, const float* W, const float* Y, long long rows, int dim,
                                 int R, float* dy, float* G, cudaStream_t st) {
    const int V = bf16 ? 8 : 4;
    const int NC = (dim + 32 * V - 1) / (32 * V);
    if (dim % V || NC > 4 || ((uintptr_t)X & 15) || rows < 1) return cudaErrorNotSupported;
    const int nc = NC <= 1 ? 1 : NC <= 2 ? 2 : 4;
    long long nb = (rows + 7) / 8;
    if (nb > 148 * 4) nb = 148 * 4;
    const int RR = (Y || dy) ? R : 1;   // ranks to cover
    float* part = nullptr;
    if (G) {
        const int rr = Y ? (R < 4 ? R : 4) : 1;
        part = (float*)workspace(WS_GEMM_P, (size_t)nb * dim * rr * sizeof(float));
        if (!part) return cudaErrorMemoryAllocation;
    }
    const size_t smem = G ? (size_t)dim * 4 * sizeof(float) : 0;
    for (int r0 = 0; r0 < RR; r0 += 4) {
        const int rc = RR - r0 < 4 ? RR - r0 : 4;
#define KMB_RP3(TT, NCV, RMV)                                                                          \
    rank_pass<TT, NCV, RMV><<<(unsigned)nb, 256, smem, st>>>((const TT*)X, W, Y, rows, dim, R, r0, rc, dy, part)
#define KMB_RP(TT, NCV)                      \
    do {                                     \
        if (rc <= 1) KMB_RP3(TT, NCV, 1);    \
        else if (rc <= 2) KMB_RP3(TT, NCV, 2); \
        else KMB_RP3(TT, NCV, 4);            \
    } while (0)
        if (bf16) {
            if (nc == 1) KMB_RP(__nv_bfloat16, 1); else if (nc == 2) KMB_RP(__nv_bfloat16, 2); else KMB_RP(__nv_bfloat16, 4);
        } else {
            if (nc == 1) KMB_RP(float, 1); else if (nc == 2) KMB_RP(float, 2); else KMB_RP(float, 4);
        }
#undef KMB_RP3
#undef KMB_RP
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        if (G) {
            const int rr = Y ? rc : 1;
            add_rank_partials<<<nblk(dim * rr, 32), 256, 0, st>>>(part, (int)nb, dim, rr, Y ? R : 1, Y ? r0 : 0, G);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            if (!Y && !dy) break;
        }
    }
    return cudaSuccess;
}

// out[row, r] = sum_j X[row, j] W[j, r]
cudaError_t rank_rows(bool bf16, const void* X, const float* W, long long rows, int dim, int R, float* out,
                      cudaStream_t st) {
    return rank_bwd(bf16, X, W, nullptr, rows, dim, R, out, nullptr, st);
}

// G[j, r] += sum_row X[row, j] Y[row, r]  (Y == nullptr: g[j] += sum_row X[row, j])
cudaError_t rank_outer(bool bf16, const void* X, const float* Y, long long rows, int dim, int R, float* G,
                       cudaStream_t st) {
    return rank_bwd(bf16, X, nullptr, Y, rows, dim, R, nullptr, G, st);
}

// dy[row, r] = sum_j X[row, j] W[j, r] (dy non-null) and G[j, r] += sum_row X[row, j] Y[row, r] (G
// non-null) in one pass over X.
cudaError_t rank_bwd(bool bf16, const void* X, const float* W, const float* Y, long long rows, int dim, int R,
                     float* dy, float* G, cudaStream_t st) {
    cudaError_t e = rank_pass_run(bf16, X, W, Y, rows, dim, R, dy, G, st);
    if (e != cudaErrorNotSupported) return e;
    // layouts rank_pass does not take: a warp per row for dy, column partials for G
    if (dy) {
        const unsigned grid = nblk(rows * 32, 256);
        for (int r0 = 0; r0 < R; r0 += 4) {
            if (bf16)
                rank_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)X, W, rows, dim, R, r0, dy);
            else
                rank_rows_kernel<float><<<grid, 256, 0, st>>>((const float*)X, W, rows, dim, R, r0, dy);
        }
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    if (!G) return cudaSuccess;
    const int RR = Y ? R : 1;
    int nchunk = (int)((rows + 1023) / 1024);
    const int dblk = (int)nblk(dim, 128);
    if ((long long)nchunk * dblk > 1184) nchunk = 1184 / dblk > 0 ? 1184 / dblk : 1;   // ~8 blocks per SM
    const long long rpc = (rows + nchunk - 1) / nchunk;
    float* part = (float*)workspace(WS_GEMM_P, (size_t)nchunk * dim * RR * sizeof(float));
    if (!part) return cudaErrorMemoryAllocation;
    dim3 grid(dblk, nchunk);
    for (int r0 = 0; r0 < RR; r0 += 4) {
        if (bf16)
            outer_partials<__nv_bfloat16><<<grid, 128, 0, st>>>((const __nv_bfloat16*)X, Y, rows, dim, R, r0, rpc,
                                                                part);
        else
            outer_partials<float><<<grid, 128, 0, st>>>((const float*)X, Y, rows, dim, R, r0, rpc, part);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const long long n = (long long)dim * RR;
    add_partials<<<nblk(n, 256), 256, 0, st>>>(part, n, nchunk, G);
    return cudaGetLastError();
}

cudaError_t col_sums(const float* X, long long rows, int dim, float* g, cudaStream_t st) {
    return rank_bwd(false, X, nullptr, nullptr, rows, dim, 1, nullptr, g, st);
}

cudaError_t out_rank(const float* x, const float* y, const float* W, long long rows, int dim, int R, float* out,
                     cudaStream_t st) {
    const size_t wbytes = (size_t)dim * R * sizeof(float);
    if (dim % 4 == 0 && !((uintptr_t)x & 15) && !((uintptr_t)out & 15) && wbytes <= 48 * 1024) {
        const int dim4 = dim / 4, tpr = dim4 < 256 ? dim4 : 256, rpi = 256 / tpr;
        long long grid = (rows + rpi - 1) / rpi;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (grid > 8LL * sms) grid = 8LL * sms;
        if (grid < 1) grid = 1;
        out_rank_f32x4<<<(unsigned)grid, 256, wbytes, st>>>((const float4*)x, y, W, rows, dim4, R, (float4*)out);
        return cudaGetLastError();
    }
    out_rank_f32<<<nblk(rows * dim, 256), 256, 0, st>>>(x, y, W, rows, dim, R, out);
    return cudaGetLastError();
}

}  // namespace kmb

using namespace kmb;

extern "C" {

int kmb_gemm_set_f32_kind(int kind) {
    if (kind < KIND_TF32X3_ || kind > KIND_SIMT_) return set_error("kmb_gemm_set_f32_kind: unknown kind");
    g_f32_kind = kind;
    return 0;
}
int kmb_gemm_get_f32_kind(void) { return g_f32_kind; }
int kmb_gemm_set_f32_flush(int ksteps) {
    return gemm_set_kflush(ksteps) ? set_error("kmb_gemm_set_f32_flush: 1 .. 64") : 0;
}
int kmb_gemm_last_path(void) { return tl_gemm_path; }

int kmb_gemm_f32(int kind, int trans, long long M, long long N, long long K, const float* A, long long lda,
                 const float* B, long long ldb, float* D, long long ldd, int accumulate, void* stream) {
    clear_error();
    if (kind < 0) kind = g_f32_kind;
    if (kind < KIND_TF32X3_ || kind > KIND_SIMT_ || M < 1 || N < 1 || K < 1 || !A || !B || !D)
        return set_error("kmb_gemm_f32: invalid arguments");
    cudaStream_t st = (cudaStream_t)stream;
    const cudaError_t e = trans ? mm_tn_kind(kind, false, M, N, K, A, lda, B, ldb, D, ldd, accumulate != 0, st)
                                : mm_nt_kind(kind, false, M, N, K, A, lda, B, ldb, D, ldd, accumulate != 0, st);
    return e == cudaSuccess ? 0 : set_cuda_error("kmb_gemm_f32", e);
}

int kmb_gemm_bf16(int trans, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, int accumulate, void* stream) {
    clear_error();
    if (M < 1 || N < 1 || K < 1 || !A || !B || !D) return set_error("kmb_gemm_bf16: invalid arguments");
    cudaStream_t st = (cudaStream_t)stream;
    const cudaError_t e = trans ? mm_tn_kind(KIND_BF16_, true, M, N, K, A, lda, B, ldb, D, ldd, accumulate != 0, st)
                                : mm_nt_kind(KIND_BF16_, true, M, N, K, A, lda, B, ldb, D, ldd, accumulate != 0, st);
    return e == cudaSuccess ? 0 : set_cuda_error("kmb_gemm_bf16", e);
}

}  // extern "C"
