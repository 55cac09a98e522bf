// block.cu -- Mamba-3 block (projections + block scan + output projection).
//
// Reference semantics: src/mamba_block.c:106-125 (projections and
// activations), :509-528 (forward), :746-773 (backward).  On the B200 the L
// per-point GEMVs of the reference become one packed GEMM over all batch rows:
// P[BL, Rt] = X[BL, dim] . Wcat^T with Wcat = [W_in; delta_proj; lambda_proj;
// W_B; W_C] (Rt = R + 2 + 2 N R rows), on the tensor cores at fp32 accuracy
// (block_gemm.cu / gemm_tc.cu: split-bf16 pieces, stage-wise fp32 accumulation;
// the parity target is the fp32 reference).  One elementwise
// epilogue applies silu / softplus+clamp / sigmoid / biases and writes the
// block-scan inputs; the backward mirrors it.  The backward is exact: it also
// produces dW_in and the projection paths of dx, which the reference skips.
#include <cuda_bf16.h>
#include <algorithm>
#include <cstring>
#include <map>
#include "kmb_common.cuh"
#include "../../include/kmamba_block.h"

namespace kmb {
void* workspace(int slot, size_t bytes);
int set_error(const char* msg);
void clear_error();
int set_cuda_error(const char* where, cudaError_t e);
enum { WS_BLK_W = 5, WS_BLK_SCRATCH = 6, WS_BLK_WBF = 7 };

struct ActLayout {
    long long BL, Rt, NR;
    size_t proj, u, dt, lam, B, C, h, Bu, y, total;  // offsets in floats
};

static ActLayout act_layout(const KMBlockConfig* c, long batch) {
    ActLayout a;
    a.BL = (long long)batch * c->L;
    a.NR = c->N * c->R;
    a.Rt = c->R + 2 + 2 * a.NR;
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o += (n + 63) & ~(size_t)63; return r; };
    a.proj = take(a.BL * a.Rt);
    // scan inputs: bf16 (half a float each) when bf16_storage
    auto in = [&](size_t n) { return take(c->bf16_storage ? (n + 1) / 2 : n); };
    a.u = in(a.BL * c->R);
    a.dt = in(a.BL);
    a.lam = in(a.BL);
    a.B = in(a.BL * a.NR);
    a.C = in(a.BL * a.NR);
    a.h = take(a.BL * c->N);
    a.Bu = take(a.BL * c->N);
    a.y = take(a.BL * c->R);
    a.total = o;
    return a;
}

__device__ __forceinline__ float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

__device__ __forceinline__ void stv(float* p, float v) { *p = v; }
__device__ __forceinline__ void stv(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ float ldv(const float* p) { return *p; }
__device__ __forceinline__ float ldv(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// The epilogues below walk blocks of 32 rows (grid-stride over blocks, 256 threads).  The per-row columns
// (u / dt / lambda and their gradients: R + 2 of them, each with an exp / log) are computed lane-parallel:
// warp k takes column k of the block's 32 rows, one row per lane, so no warp carries them alone.  The wide
// parts (B / C and their gradients) are copied by all threads as coalesced row segments, four rows in flight.
constexpr int EPI_RB = 32;

// Forward epilogue over P[BL, Rt]; T = storage type of the scan inputs.
template <typename T>
__global__ void __launch_bounds__(256) block_fwd_epilogue(const float* __restrict__ P, long long BL, int R, int NR,
                                                          float dt_min, float dt_max, const float* __restrict__ bB,
                                                          const float* __restrict__ bC, T* __restrict__ u,
                                                          T* __restrict__ dt, T* __restrict__ lam, T* __restrict__ B,
                                                          T* __restrict__ C) {
    const int Rt = R + 2 + 2 * NR;
    const int tpr = NR < 256 ? NR : 256, rpi = 256 / tpr;
    const int sub = threadIdx.x / tpr, c0 = threadIdx.x - sub * tpr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (long long r0 = (long long)blockIdx.x * EPI_RB; r0 < BL; r0 += (long long)gridDim.x * EPI_RB) {
        const int nrow = BL - r0 < EPI_RB ? (int)(BL - r0) : EPI_RB;
        if (sub < rpi) {
#pragma unroll 4
            for (int rr = sub; rr < nrow; rr += rpi) {
                const long long row = r0 + rr;
                const float* pr = P + row * Rt + R + 2;
                for (int j = c0; j < NR; j += tpr) {
                    stv(B + row * NR + j, pr[j] + bB[j]);
                    stv(C + row * NR + j, pr[NR + j] + bC[j]);
                }
            }
        }
        if (lane < nrow) {
            const long long row = r0 + lane;
            for (int j = warp; j < R + 2; j += 8) {
                const float v = P[row * Rt + j];
                if (j < R) {
                    stv(u + row * R + j, v / (1.0f + expf(-v)));          // silu
                } else if (j == R) {
                    float d = logf(1.0f + expf(v));                         // softplus
                    if (d < dt_min) d = dt_min;
                    if (d > dt_max) d = dt_max;
                    stv(dt + row, d);
                } else {
                    stv(lam + row, sigm(v));
                }
            }
        }
    }
}

// Gradient of the per-row column j < R + 2 of P (silu', softplus' inside the clamp, sigmoid')
template <typename T>
__device__ __forceinline__ float epi_grad_col(const float* __restrict__ P, const T* __restrict__ lamv, long long row,
                                              int Rt, int R, int j, float dt_min, float dt_max,
                                              const float* __restrict__ du, const float* __restrict__ ddt,
                                              const float* __restrict__ dlam) {
    if (j < R) {
        const float z = P[row * Rt + j], s = sigm(z);
        return du[row * R + j] * s * (1.0f + z * (1.0f - s));
    }
    if (j == R) {
        // clamp test on the unrounded softplus (identical to the stored dt in fp32 mode)
        const float z = P[row * Rt + j];
        const float d = fminf(fmaxf(logf(1.0f + expf(z)), dt_min), dt_max);
        return (d > dt_min && d < dt_max) ? ddt[row] * sigm(z) : 0.0f;
    }
    const float l = ldv(lamv + row);
    return dlam[row] * l * (1.0f - l);
}

// Backward epilogue: dP[BL, Rt] from the scan gradients (O = float, or bf16
// as the operand of the bf16 tensor-core gradient GEMMs).  dP rows have ldo >= Rt
// columns; columns Rt .. ldo-1 are written as zero.
template <typename T, typename O>
__global__ void __launch_bounds__(256) block_bwd_epilogue(const float* __restrict__ P, const T* __restrict__ dtv,
                                                          const T* __restrict__ lamv, long long BL, int R, int NR,
                                                          float dt_min, float dt_max, const float* __restrict__ du,
                                                          const float* __restrict__ ddt,
                                                          const float* __restrict__ dlam,
                                                          const float* __restrict__ dB,
                                                          const float* __restrict__ dC, O* __restrict__ dP,
                                                          int ldo) {
    const int Rt = R + 2 + 2 * NR, pad = ldo - Rt;
    const int W = NR > pad ? NR : pad;
    const int tpr = W < 256 ? W : 256, rpi = 256 / tpr;
    const int sub = threadIdx.x / tpr, c0 = threadIdx.x - sub * tpr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    (void)dtv;
    for (long long r0 = (long long)blockIdx.x * EPI_RB; r0 < BL; r0 += (long long)gridDim.x * EPI_RB) {
        const int nrow = BL - r0 < EPI_RB ? (int)(BL - r0) : EPI_RB;
        if (sub < rpi) {
#pragma unroll 4
            for (int rr = sub; rr < nrow; rr += rpi) {
                const long long row = r0 + rr;
                O* dr = dP + row * ldo;
                for (int j = c0; j < W; j += tpr) {
                    if (j < NR) {
                        stv(dr + R + 2 + j, dB[row * NR + j]);
                        stv(dr + R + 2 + NR + j, dC[row * NR + j]);
                    }
                    if (j < pad) stv(dr + Rt + j, 0.0f);
                }
            }
        }
        if (lane < nrow) {
            const long long row = r0 + lane;
            for (int j = warp; j < R + 2; j += 8)
                stv(dP + row * ldo + j, epi_grad_col(P, lamv, row, Rt, R, j, dt_min, dt_max, du, ddt, dlam));
        }
    }
}

// The bf16 form of block_bwd_epilogue: 8 consecutive dP columns per thread (one 16-byte store);
// ldo % 8 == 0 and a 16-byte-aligned dP.  The chunks holding per-row columns (the first
// ceil((R + 2) / 8)) are computed lane-parallel (warp k: chunk k of the block's rows, a row per lane);
// the others are copies.  Same per-element arithmetic.
template <typename T>
__global__ void __launch_bounds__(256) block_bwd_epilogue_v8(const float* __restrict__ P,
                                                             const T* __restrict__ lamv, long long BL, int R,
                                                             int NR, float dt_min, float dt_max,
                                                             const float* __restrict__ du,
                                                             const float* __restrict__ ddt,
                                                             const float* __restrict__ dlam,
                                                             const float* __restrict__ dB,
                                                             const float* __restrict__ dC,
                                                             __nv_bfloat16* __restrict__ dP, int ldo) {
    const int Rt = R + 2 + 2 * NR, ch = ldo >> 3, nsc = (R + 2 + 7) >> 3;
    const int W = ch - nsc;   // copy chunks per row
    const int tpr = W < 256 ? (W < 1 ? 1 : W) : 256, rpi = 256 / tpr;
    const int sub = threadIdx.x / tpr, k0 = threadIdx.x - sub * tpr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto chunk = [&](long long row, int c0, bool special) {
        uint4 pk;
        __nv_bfloat16* e = (__nv_bfloat16*)&pk;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int col = c0 + j;
            float g;
            if (col >= Rt) g = 0.0f;
            else if (col >= R + 2) g = col < R + 2 + NR ? dB[row * NR + (col - R - 2)] : dC[row * NR + (col - R - 2 - NR)];
            else g = special ? epi_grad_col(P, lamv, row, Rt, R, col, dt_min, dt_max, du, ddt, dlam) : 0.0f;
            e[j] = __float2bfloat16_rn(g);
        }
        *(uint4*)(dP + row * ldo + c0) = pk;
    };
    for (long long r0 = (long long)blockIdx.x * EPI_RB; r0 < BL; r0 += (long long)gridDim.x * EPI_RB) {
        const int nrow = BL - r0 < EPI_RB ? (int)(BL - r0) : EPI_RB;
        if (sub < rpi && W > 0) {
#pragma unroll 2
            for (int rr = sub; rr < nrow; rr += rpi)
                for (int k = nsc + k0; k < ch; k += tpr) chunk(r0 + rr, k * 8, false);
        }
        if (lane < nrow)
            for (int k = warp; k < nsc; k += 8) chunk(r0 + lane, k * 8, true);
    }
}

// grads += slices of G[Rt, dim]
__global__ void block_scatter_grads(const float* __restrict__ G, int R, int NR, int dim, float* gWin,
                                    float* gdelta, float* glam, float* gWB, float* gWC) {
    const long long Rt = R + 2 + 2LL * NR;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= Rt * dim) return;
    const int row = (int)(i / dim), col = (int)(i - (long long)row * dim);
    const float v = G[i];
    float* dst;
    if (row < R) dst = gWin ? gWin + (long long)row * dim : nullptr;
    else if (row == R) dst = gdelta;
    else if (row == R + 1) dst = glam;
    else if (row < R + 2 + NR) dst = gWB ? gWB + (long long)(row - R - 2) * dim : nullptr;
    else dst = gWC ? gWC + (long long)(row - R - 2 - NR) * dim : nullptr;
    if (dst) dst[col] += v;
}

__global__ void to_bf16(const float* __restrict__ a, __nv_bfloat16* __restrict__ b, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b[i] = __float2bfloat16_rn(a[i]);
}
// out[row, d] = bf16(x[row, d] + sum_r y[row, r] W_out[d, r])   (bf16 residual stream).
// A thread owns an 8-channel column chunk (16 bytes), keeps its W_out slice in
// registers and walks rows; dim % 8 == 0, 16-byte aligned x / out, R <= RM.
template <int RM>
__global__ void block_out_bf16_cols(const uint4* __restrict__ x, const float* __restrict__ y,
                                    const float* __restrict__ Wout, long long rows, int dim8, int R,
                                    uint4* __restrict__ out) {
    const int c = threadIdx.x % dim8, rpb = blockDim.x / dim8;
    const int d0 = c * 8;
    if ((int)threadIdx.x >= rpb * dim8) return;
    float w[8][RM];
#pragma unroll
    for (int e = 0; e < 8; e++)
#pragma unroll
        for (int r = 0; r < RM; r++) w[e][r] = r < R ? Wout[(long long)(d0 + e) * R + r] : 0.0f;
    for (long long row = (long long)blockIdx.x * rpb + threadIdx.x / dim8; row < rows; row += (long long)gridDim.x * rpb) {
        float yr[RM];
#pragma unroll
        for (int r = 0; r < RM; r++) yr[r] = r < R ? y[row * R + r] : 0.0f;
        const long long i = row * dim8 + c;
        uint4 xv = x[i];
        __nv_bfloat16* xe = (__nv_bfloat16*)&xv;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float acc = 0.0f;
#pragma unroll
            for (int r = 0; r < RM; r++) acc = __fmaf_rn(yr[r], w[e][r], acc);
            xe[e] = __float2bfloat16_rn(__bfloat162float(xe[e]) + acc);
        }
        out[i] = xv;
    }
}
__global__ void block_out_bf16(const __nv_bfloat16* __restrict__ x, const float* __restrict__ y,
                               const float* __restrict__ Wout, long long BL, int dim, int R,
                               __nv_bfloat16* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= BL * dim) return;
    const long long row = i / dim;
    const int d = (int)(i - row * dim);
    float acc = 0.0f;
    for (int r = 0; r < R; r++) acc = __fmaf_rn(y[row * R + r], Wout[(long long)d * R + r], acc);
    out[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + acc);
}

__global__ void sub_inplace(float* __restrict__ y, const float* __restrict__ x, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] -= x[i];
}

int* device_status();
cudaError_t launch_proj_fwd_tc(const __nv_bfloat16* X, const float* Win, const float* dp, const float* lp,
                               const float* WB, const float* WC, __nv_bfloat16* W, long long BL, int dim, int R,
                               int NR, float dt_min, float dt_max, const float* bB, const float* bC, float* P,
                               __nv_bfloat16* u, __nv_bfloat16* dt, __nv_bfloat16* lam, __nv_bfloat16* B,
                               __nv_bfloat16* C, int* status, cudaStream_t st);
// 1: route the bf16 projections through the plain tensor-core GEMM + separate epilogues (tests / comparison)
static thread_local int tl_no_tc = 0;
static thread_local int tl_proj_path = -1;  // projection of the last bf16 forward: 1 fused tensor-core kernel, 0 plain GEMM
static thread_local int tl_dx_path = -1;    // dx GEMM of the last bf16 backward: 1 fused tensor-core kernel, 0 plain GEMM
cudaError_t launch_dx_tc(const __nv_bfloat16* dP, int ldp, const float* Win, const float* dp, const float* lp,
                         const float* WB, const float* WC, __nv_bfloat16* Wt, long long BL, int dim, int R, int NR,
                         const __nv_bfloat16* dout, __nv_bfloat16* dx, int* status, cudaStream_t st);

// matrix products of the block (block_gemm.cu): tensor cores for the large ones, own kernels for rank R
cudaError_t mm_nt(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st);
cudaError_t mm_nt_same_a(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                         long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st);
cudaError_t mm_tn(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st);
cudaError_t rank_rows(bool bf16, const void* X, const float* W, long long rows, int dim, int R, float* out,
                      cudaStream_t st);
cudaError_t rank_outer(bool bf16, const void* X, const float* Y, long long rows, int dim, int R, float* G,
                       cudaStream_t st);
cudaError_t col_sums(const float* X, long long rows, int dim, float* g, cudaStream_t st);
cudaError_t rank_bwd(bool bf16, const void* X, const float* W, const float* Y, long long rows, int dim, int R,
                     float* dy, float* G, cudaStream_t st);
cudaError_t out_rank(const float* x, const float* y, const float* W, long long rows, int dim, int R, float* out,
                     cudaStream_t st);
cudaError_t gemm_transpose_f32(const float* in, float* out, long long R, long long Cn, long long ldi, long long ldo,
                               cudaStream_t st);
cudaError_t launch_pack_wcat_t(const float* Win, const float* dp, const float* lp, const float* WB, const float* WC,
                               int R, int NR, int dim, int ldp, __nv_bfloat16* out, cudaStream_t st);

static inline unsigned nb(long long n, int t) { return (unsigned)((n + t - 1) / t); }

// Grid of the epilogues: one CTA per 32-row block, at most 8 CTAs of 256 threads per SM (grid-stride)
static unsigned epi_grid(long long rows) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    }
    long long g = (rows + EPI_RB - 1) / EPI_RB;
    if (g > 8LL * sms) g = 8LL * sms;
    return (unsigned)(g < 1 ? 1 : g);
}

static int check_cfg(const KMBlockConfig* c, const KMBlockWeights* w, long batch) {
    if (!c || !w || batch < 1 || c->dim < 1 || c->N < 1 || c->N > 64 || c->R < 1 || c->L < 1)
        return set_error("invalid KMBlockConfig (N must be 1..64)");
    if (!w->W_in || !w->W_out || !w->A_log || !w->W_B || !w->W_C || !w->delta_proj || !w->lambda_proj ||
        !w->b_B || !w->b_C || !w->theta)
        return set_error("KMBlockWeights: every parameter pointer is required");
    return 0;
}

// Wcat = [W_in; delta_proj; lambda_proj; W_B; W_C]  [Rt, dim]
static float* pack_wcat(const KMBlockConfig* c, const KMBlockWeights* w, cudaStream_t st) {
    const long long NR = c->N * c->R, Rt = c->R + 2 + 2 * NR, dim = c->dim;
    float* W = (float*)workspace(WS_BLK_W, (size_t)Rt * dim * sizeof(float));
    if (!W) return nullptr;
    const float* src[5] = {w->W_in, w->delta_proj, w->lambda_proj, w->W_B, w->W_C};
    const long long rows[5] = {c->R, 1, 1, NR, NR};
    long long r0 = 0;
    for (int i = 0; i < 5; i++) {
        if (cudaMemcpyAsync(W + r0 * dim, src[i], (size_t)rows[i] * dim * sizeof(float), cudaMemcpyDeviceToDevice,
                            st) != cudaSuccess)
            return nullptr;
        r0 += rows[i];
    }
    return W;
}

}  // namespace kmb

using namespace kmb;

extern "C" size_t kmb_block_activation_floats(const KMBlockConfig* c, long batch) {
    if (!c || batch < 1) return 0;
    return act_layout(c, batch).total;
}

extern "C" void kmb_block_set_tensor_cores(int on) { tl_no_tc = on ? 0 : 1; }
extern "C" int kmb_block_last_projection_path(void) { return tl_proj_path; }
extern "C" int kmb_block_last_dx_path(void) { return tl_dx_path; }

extern "C" int kmb_block_forward(const KMBlockConfig* c, const KMBlockWeights* w, const float* x, float* out,
                                 long batch, float* act, void* stream) {
    if (check_cfg(c, w, batch)) return -1;
    if (!x || !out || !act) return set_error("kmb_block_forward: x, out, act required");
    cudaStream_t st = (cudaStream_t)stream;
    const ActLayout a = act_layout(c, batch);
    float* W = pack_wcat(c, w, st);
    if (!W) return set_error("kmb_block_forward: weight packing failed");
    const int dim = (int)c->dim;
    const bool bf = c->bf16_storage != 0;
    cudaError_t e;
    if (bf) {
        // bf16 x bf16 -> fp32 projection GEMM on the tensor cores
        __nv_bfloat16* Wb = (__nv_bfloat16*)workspace(WS_BLK_WBF, (size_t)a.Rt * dim * sizeof(__nv_bfloat16));
        if (!Wb) return set_error("workspace allocation failed");
        typedef __nv_bfloat16 H;
        // tensor-core projection with the epilogue fused (tcgen05); the plain tensor-core GEMM + epilogue otherwise
        int* status = device_status();
        if (status && !tl_no_tc) {
            cudaMemsetAsync(status, 0, sizeof(int), st);
            e = launch_proj_fwd_tc((const H*)x, w->W_in, w->delta_proj, w->lambda_proj, w->W_B, w->W_C, Wb, a.BL,
                                   dim, (int)c->R, (int)a.NR, c->dt_min, c->dt_max, w->b_B, w->b_C, act + a.proj,
                                   (H*)(act + a.u), (H*)(act + a.dt), (H*)(act + a.lam), (H*)(act + a.B),
                                   (H*)(act + a.C), status, st);
            if (e != cudaSuccess && e != cudaErrorNotSupported) return set_cuda_error("tensor-core projection", e);
        } else {
            e = cudaErrorNotSupported;
        }
        tl_proj_path = e == cudaSuccess ? 1 : 0;
        if (e == cudaSuccess) goto scan;
        cudaGetLastError();
        to_bf16<<<nb(a.Rt * dim, 256), 256, 0, st>>>(W, Wb, a.Rt * dim);
        if ((e = mm_nt(true, a.BL, a.Rt, dim, x, dim, Wb, dim, act + a.proj, a.Rt, false, st)) != cudaSuccess)
            return set_cuda_error("bf16 projection GEMM", e);
        block_fwd_epilogue<H><<<epi_grid(a.BL), 256, 0, st>>>(
            act + a.proj, a.BL, (int)c->R, (int)a.NR, c->dt_min, c->dt_max, w->b_B, w->b_C, (H*)(act + a.u),
            (H*)(act + a.dt), (H*)(act + a.lam), (H*)(act + a.B), (H*)(act + a.C));
    } else {
        // P[BL, Rt] = X[BL, dim] . Wcat^T on the tensor cores at fp32 accuracy (3xTF32)
        if ((e = mm_nt(false, a.BL, a.Rt, dim, x, dim, W, dim, act + a.proj, a.Rt, false, st)) != cudaSuccess)
            return set_cuda_error("projection GEMM", e);
        block_fwd_epilogue<float><<<epi_grid(a.BL), 256, 0, st>>>(
            act + a.proj, a.BL, (int)c->R, (int)a.NR, c->dt_min, c->dt_max, w->b_B, w->b_C, act + a.u, act + a.dt,
            act + a.lam, act + a.B, act + a.C);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("block epilogue", e);
scan:
    KMBlockScanParams p;
    memset(&p, 0, sizeof p);
    p.ndims = c->ndims; p.dims = c->dims; p.L = c->L; p.N = c->N; p.R = c->R;
    p.u = act + a.u; p.dt = act + a.dt; p.lambda = act + a.lam; p.B = act + a.B; p.C = act + a.C;
    p.A_log = w->A_log; p.theta = w->theta; p.default_lambda = c->default_lambda; p.use_fast_exp = c->use_fast_exp;
    p.h = act + a.h; p.Bu = act + a.Bu; p.y = act + a.y;
    p.inputs_bf16 = bf;
    if (kmb_blockscan_forward(&p, batch, stream)) return -1;
    if (bf) {
        const int dim8 = dim / 8;
        if (dim % 8 == 0 && dim8 <= 256 && c->R <= 4 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0) {
            const int rpb = 256 / dim8;
            const unsigned grid = (unsigned)std::min<long long>((a.BL + rpb - 1) / rpb, 148LL * 8);
            if (c->R <= 2)
                block_out_bf16_cols<2><<<grid, 256, 0, st>>>((const uint4*)x, act + a.y, w->W_out, a.BL, dim8,
                                                             (int)c->R, (uint4*)out);
            else
                block_out_bf16_cols<4><<<grid, 256, 0, st>>>((const uint4*)x, act + a.y, w->W_out, a.BL, dim8,
                                                             (int)c->R, (uint4*)out);
        } else
            block_out_bf16<<<nb(a.BL * dim, 256), 256, 0, st>>>((const __nv_bfloat16*)x, act + a.y, w->W_out, a.BL,
                                                               dim, (int)c->R, (__nv_bfloat16*)out);
        e = cudaGetLastError();
        return e == cudaSuccess ? 0 : set_cuda_error("bf16 output", e);
    }
    // out = x + y . W_out^T (rank R: one elementwise pass)
    if ((e = out_rank(x, act + a.y, w->W_out, a.BL, dim, (int)c->R, out, st)) != cudaSuccess)
        return set_cuda_error("output projection", e);
    return 0;
}

// fp32-storage backward
static int block_backward_f32(const KMBlockConfig* c, const KMBlockWeights* w, const float* x, const float* dout,
                              float* dx, const KMBlockGrads* g, long batch, const float* act, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    const ActLayout a = act_layout(c, batch);
    const int dim = (int)c->dim, R = (int)c->R;
    const long long BL = a.BL, NR = a.NR, Rt = a.Rt;
    // scratch: dy[BL,R] | du[BL,R] | ddt[BL] | dlam[BL] | dB[BL,NR] | dC[BL,NR] | dP[BL,Rt] | G[Rt,dim] | Wcat^T
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o += (n + 63) & ~(size_t)63; return r; };
    const size_t s_dy = take(BL * R), s_du = take(BL * R), s_ddt = take(BL), s_dlam = take(BL);
    const long long ldq = (Rt + 3) & ~3LL;   // dP and Wcat^T row stride: 16-byte rows for the tensor-core loads
    const size_t s_dB = take(BL * NR), s_dC = take(BL * NR), s_dP = take(BL * ldq), s_G = take(Rt * dim);
    const size_t s_WT = take((size_t)dim * ldq);
    float* S = (float*)workspace(WS_BLK_SCRATCH, o * sizeof(float));
    if (!S) return set_error("workspace allocation failed");
    float* W = pack_wcat(c, w, st);
    if (!W) return set_error("kmb_block_backward: weight packing failed");
    cudaError_t e;
    // d_y[BL,R] = dout . W_out ; gW_out += dout^T . y   (rank R, one pass over dout)
    if ((e = rank_bwd(false, dout, w->W_out, act + a.y, BL, dim, R, S + s_dy, g->W_out, st)) != cudaSuccess)
        return set_cuda_error("dy / dW_out", e);
    KMBlockScanParams p;
    memset(&p, 0, sizeof p);
    p.ndims = c->ndims; p.dims = c->dims; p.L = c->L; p.N = c->N; p.R = c->R;
    p.u = act + a.u; p.dt = act + a.dt; p.lambda = act + a.lam; p.B = act + a.B; p.C = act + a.C;
    p.A_log = w->A_log; p.theta = w->theta; p.default_lambda = c->default_lambda; p.use_fast_exp = c->use_fast_exp;
    p.h = (float*)(act + a.h); p.Bu = (float*)(act + a.Bu); p.y = (float*)(act + a.y);
    KMBlockScanGrads sg;
    sg.dB = S + s_dB; sg.dC = S + s_dC; sg.du = S + s_du; sg.ddt = S + s_ddt; sg.dlambda = S + s_dlam;
    sg.dA_log = g->A_log; sg.dtheta = g->theta;
    // du, ddt, dlambda, dB, dC are assigned (no clearing of the scratch first)
    if (kmb_blockscan_backward_ex(&p, batch, S + s_dy, &sg, 1, stream)) return -1;
    block_bwd_epilogue<float, float><<<epi_grid(BL), 256, 0, st>>>(act + a.proj, act + a.dt, act + a.lam, BL, R,
                                                                     (int)NR, c->dt_min, c->dt_max, S + s_du,
                                                                     S + s_ddt, S + s_dlam, S + s_dB, S + s_dC,
                                                                     S + s_dP, (int)ldq);
    if ((e = cudaGetLastError()) != cudaSuccess) return set_cuda_error("block bwd epilogue", e);
    // G[Rt, dim] = dP^T . X (tensor cores, K = BL split over the SMs) -> scatter into the projection gradients
    if ((e = mm_tn(false, Rt, dim, BL, S + s_dP, ldq, x, dim, S + s_G, dim, false, st)) != cudaSuccess)
        return set_cuda_error("dWcat GEMM", e);
    block_scatter_grads<<<nb(Rt * dim, 256), 256, 0, st>>>(S + s_G, R, (int)NR, dim, g->W_in, g->delta_proj,
                                                           g->lambda_proj, g->W_B, g->W_C);
    if ((e = cudaGetLastError()) != cudaSuccess) return set_cuda_error("grad scatter", e);
    // bias gradients: column sums of dB, dC (+= into the gradients)
    if (g->b_B && (e = col_sums(S + s_dB, BL, (int)NR, g->b_B, st)) != cudaSuccess) return set_cuda_error("db_B", e);
    if (g->b_C && (e = col_sums(S + s_dC, BL, (int)NR, g->b_C, st)) != cudaSuccess) return set_cuda_error("db_C", e);
    if (dx) {
        // dx may alias dout (the reference model passes one buffer for both): dout is last read above
        if (dx != dout && (e = cudaMemcpyAsync(dx, dout, (size_t)BL * dim * sizeof(float), cudaMemcpyDeviceToDevice, st)) !=
            cudaSuccess)
            return set_cuda_error("dx copy", e);
        // dx += dP[BL, Rt] . Wcat[Rt, dim]: the B operand is Wcat^T [dim, Rt] (row stride ldq; the loads
        // past column Rt read zeros)
        if ((e = gemm_transpose_f32(W, S + s_WT, Rt, dim, dim, ldq, st)) != cudaSuccess)
            return set_cuda_error("Wcat^T", e);
        // dP's pieces from the dWcat product above are still in the workspace: not split again
        if ((e = mm_nt_same_a(false, BL, dim, Rt, S + s_dP, ldq, S + s_WT, ldq, dx, dim, true, st)) != cudaSuccess)
            return set_cuda_error("dx GEMM", e);
    }
    return 0;
}

// dx = bf16(dout + D)   (bf16 residual stream; dx may alias dout), 8 elements per thread
__global__ void residual_bf16(const __nv_bfloat16* dout, const float* __restrict__ D, __nv_bfloat16* dx, long long n) {
    const long long i8 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (i8 + 8 <= n && (((uintptr_t)dout | (uintptr_t)dx) & 15) == 0 && ((uintptr_t)D & 15) == 0) {
        uint4 v = *(const uint4*)(dout + i8);
        const float4 a = *(const float4*)(D + i8), b = *(const float4*)(D + i8 + 4);
        __nv_bfloat16* e = (__nv_bfloat16*)&v;
        const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; j++) e[j] = __float2bfloat16_rn(__bfloat162float(e[j]) + f[j]);
        *(uint4*)(dx + i8) = v;
    } else {
        for (long long i = i8; i < i8 + 8 && i < n; i++) dx[i] = __float2bfloat16_rn(__bfloat162float(dout[i]) + D[i]);
    }
}

// bf16-storage backward: x, dout, dx bf16; dWcat and dx run as bf16 x bf16 ->
// fp32 on the tensor cores (dP rounded to bf16), the rank-R products (dy, dW_out)
// read the bf16 dout with fp32 y and W_out; the scan backward and every
// gradient accumulate in fp32.
static int block_backward_bf16(const KMBlockConfig* c, const KMBlockWeights* w, const __nv_bfloat16* x,
                               const __nv_bfloat16* dout, __nv_bfloat16* dx, const KMBlockGrads* g, long batch,
                               const float* act, void* stream) {
    typedef __nv_bfloat16 H;
    cudaStream_t st = (cudaStream_t)stream;
    const ActLayout a = act_layout(c, batch);
    const int dim = (int)c->dim, R = (int)c->R;
    const long long BL = a.BL, NR = a.NR, Rt = a.Rt;
    // scratch (floats): dy | du | ddt | dlam | dB | dC | G[Rt,dim] | ones | D[BL,dim] | bf16: dP | y | W_out | Wcat
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o += (n + 63) & ~(size_t)63; return r; };
    const size_t s_dy = take(BL * R), s_du = take(BL * R), s_ddt = take(BL), s_dlam = take(BL);
    const size_t s_dB = take(BL * NR), s_dC = take(BL * NR), s_G = take(Rt * dim), s_one = take(BL);
    const int ldp = (int)((Rt + 15) & ~15LL);   // dP row stride (16-byte rows, zero padding) for TMA
    const size_t s_D = dx ? take(BL * dim) : 0;
    const size_t s_dP = take((BL * ldp + 1) / 2), s_yb = take((BL * R + 1) / 2), s_wo = take((dim * R + 1) / 2);
    const size_t s_wb = take(((size_t)ldp * dim + 1) / 2);
    float* S = (float*)workspace(WS_BLK_SCRATCH, o * sizeof(float));
    if (!S) return set_error("workspace allocation failed");
    H *dPb = (H*)(S + s_dP), *yb = (H*)(S + s_yb), *wob = (H*)(S + s_wo), *Wb = (H*)(S + s_wb);
    cudaError_t e;
    (void)yb;
    (void)wob;
    // d_y[BL,R] = dout . W_out ; gW_out += dout^T . y   (rank R, one pass over dout)
    if ((e = rank_bwd(true, dout, w->W_out, act + a.y, BL, dim, R, S + s_dy, g->W_out, st)) != cudaSuccess)
        return set_cuda_error("dy / dW_out", e);
    KMBlockScanParams p;
    memset(&p, 0, sizeof p);
    p.ndims = c->ndims; p.dims = c->dims; p.L = c->L; p.N = c->N; p.R = c->R;
    p.u = act + a.u; p.dt = act + a.dt; p.lambda = act + a.lam; p.B = act + a.B; p.C = act + a.C;
    p.A_log = w->A_log; p.theta = w->theta; p.default_lambda = c->default_lambda; p.use_fast_exp = c->use_fast_exp;
    p.h = (float*)(act + a.h); p.Bu = (float*)(act + a.Bu); p.y = (float*)(act + a.y);
    p.inputs_bf16 = 1;
    KMBlockScanGrads sg;
    sg.dB = S + s_dB; sg.dC = S + s_dC; sg.du = S + s_du; sg.ddt = S + s_ddt; sg.dlambda = S + s_dlam;
    sg.dA_log = g->A_log; sg.dtheta = g->theta;
    // du, ddt, dlambda, dB, dC are assigned (no clearing of the scratch first)
    if (kmb_blockscan_backward_ex(&p, batch, S + s_dy, &sg, 1, stream)) return -1;
    // ldp is a multiple of 16 and dPb 256-byte aligned: the 8-column form applies
    block_bwd_epilogue_v8<H><<<epi_grid(BL), 256, 0, st>>>(
        act + a.proj, (const H*)(act + a.lam), BL, R, (int)NR, c->dt_min, c->dt_max, S + s_du, S + s_ddt,
        S + s_dlam, S + s_dB, S + s_dC, dPb, ldp);
    if ((e = cudaGetLastError()) != cudaSuccess) return set_cuda_error("block bwd epilogue", e);
    // G[Rt, dim] = dP^T . X (tensor cores, K = BL split over the SMs) -> scatter into the projection gradients
    if ((e = mm_tn(true, Rt, dim, BL, dPb, ldp, x, dim, S + s_G, dim, false, st)) != cudaSuccess)
        return set_cuda_error("dWcat GEMM", e);
    block_scatter_grads<<<nb(Rt * dim, 256), 256, 0, st>>>(S + s_G, R, (int)NR, dim, g->W_in, g->delta_proj,
                                                           g->lambda_proj, g->W_B, g->W_C);
    if ((e = cudaGetLastError()) != cudaSuccess) return set_cuda_error("grad scatter", e);
    (void)s_one;
    if (g->b_B && (e = col_sums(S + s_dB, BL, (int)NR, g->b_B, st)) != cudaSuccess) return set_cuda_error("db_B", e);
    if (g->b_C && (e = col_sums(S + s_dC, BL, (int)NR, g->b_C, st)) != cudaSuccess) return set_cuda_error("db_C", e);
    if (dx) {
        // dx = dout + dP Wcat: tensor cores with the residual fused (tcgen05), else the plain tensor-core GEMM
        // and a residual kernel
        int* status = device_status();
        if (status && !tl_no_tc) {
            cudaMemsetAsync(status, 0, sizeof(int), st);
            e = launch_dx_tc(dPb, ldp, w->W_in, w->delta_proj, w->lambda_proj, w->W_B, w->W_C, Wb, BL, dim, R,
                             (int)NR, dout, dx, status, st);
            if (e != cudaSuccess && e != cudaErrorNotSupported) return set_cuda_error("tensor-core dx", e);
        } else {
            e = cudaErrorNotSupported;
        }
        tl_dx_path = e == cudaSuccess ? 1 : 0;
        if (e != cudaSuccess) {
            cudaGetLastError();
            // Wt = Wcat^T [dim, ldp] bf16 (zero columns past Rt), then D[BL, dim] = dP . Wt^T
            if ((e = launch_pack_wcat_t(w->W_in, w->delta_proj, w->lambda_proj, w->W_B, w->W_C, R, (int)NR, dim, ldp,
                                        Wb, st)) != cudaSuccess)
                return set_cuda_error("Wcat^T", e);
            if ((e = mm_nt(true, BL, dim, ldp, dPb, ldp, Wb, ldp, S + s_D, dim, false, st)) != cudaSuccess)
                return set_cuda_error("dx GEMM", e);
            residual_bf16<<<nb((BL * dim + 7) / 8, 256), 256, 0, st>>>(dout, S + s_D, dx, BL * dim);
        }
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("bf16 backward", e);
}

extern "C" int kmb_block_backward(const KMBlockConfig* c, const KMBlockWeights* w, const float* x,
                                  const float* dout, float* dx, const KMBlockGrads* g, long batch, const float* act,
                                  void* stream) {
    if (check_cfg(c, w, batch)) return -1;
    if (!x || !dout || !act || !g) return set_error("kmb_block_backward: x, dout, act, g required");
    if (!c->bf16_storage) return block_backward_f32(c, w, x, dout, dx, g, batch, act, stream);
    return block_backward_bf16(c, w, (const __nv_bfloat16*)x, (const __nv_bfloat16*)dout, (__nv_bfloat16*)dx, g,
                               batch, act, stream);
}

// ---------------------------------------------------------------------------
// The reference's cuda_block_forward / cuda_block_backward signatures, served by
// the kernels above.  The packed activation buffer is rebuilt from / copied to
// the caller's named workspace buffers (one sequence per call, like the
// reference).
namespace {
__global__ void gather_proj(const float* P, long long L, int Rt, int R, float* u_raw, float* dt_raw, float* lam_raw) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= L) return;
    for (int r = 0; r < R; r++) u_raw[t * R + r] = P[t * Rt + r];
    dt_raw[t] = P[t * Rt + R];
    lam_raw[t] = P[t * Rt + R + 1];
}
__global__ void scatter_proj(float* P, long long L, int Rt, int R, int NR, const float* u_raw, const float* dt_raw,
                             const float* lam_raw, const float* Bx, const float* Cx) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= L) return;
    for (int r = 0; r < R; r++) P[t * Rt + r] = u_raw[t * R + r];
    P[t * Rt + R] = dt_raw[t];
    P[t * Rt + R + 1] = lam_raw ? lam_raw[t] : 0.0f;
    for (int j = 0; j < NR; j++) {
        P[t * Rt + R + 2 + j] = Bx[t * NR + j];
        P[t * Rt + R + 2 + NR + j] = Cx[t * NR + j];
    }
}

// Bu[t, n] = sum_r B[t, r N + n] u[t, r] in the forward scan's fma order, for callers that keep
// no copy of it (the reference passes NULL for dt_exp).
__global__ void rebuild_bu(const float* B, const float* u, long long L, int N, int R, float* Bu) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L * N) return;
    const long long t = i / N;
    const int n = (int)(i - t * N);
    float acc = 0.0f;
    for (int r = 0; r < R; r++) acc = __fmaf_rn(B[t * (long long)N * R + r * N + n], u[t * R + r], acc);
    Bu[i] = acc;
}

KMBlockConfig ref_cfg(int L, int state, int dim, int R, int nd, const long* dims) {
    KMBlockConfig c;
    memset(&c, 0, sizeof c);
    c.dim = dim; c.N = state; c.R = R < 1 ? 1 : R; c.ndims = nd; c.dims = dims; c.L = L;
    c.dt_min = 0.001f; c.dt_max = 0.1f; c.default_lambda = 0.5f;  // reference GPU kernels hard-code these
    return c;
}
}  // namespace

extern "C" void cuda_block_forward(void* cublas, const float* d_W_in, const float* d_W_out, const float* d_A_log,
                                   const float* d_W_B, const float* d_W_C, const float* d_delta_proj,
                                   const float* d_theta, const float* d_lambda_proj, const float* d_x, float* d_y,
                                   float* d_u_raw, float* d_u, float* d_dt_raw, float* d_dt, float* d_B_exp,
                                   float* d_C_exp, float* d_dt_exp, float* d_h_store, float* d_y_scan,
                                   float* d_y_proj, float* d_lambda_raw, float* d_lambda, int L, int state, int dim,
                                   int R, int spatial_ndims, const long* spatial_dims) {
    (void)cublas;
    clear_error();
    KMBlockConfig c = ref_cfg(L, state, dim, R, spatial_ndims, spatial_dims);
    const long long NR = (long long)state * c.R;
    float* zeros = (float*)workspace(WS_BLK_WBF + 2, (size_t)NR * sizeof(float) * 2);
    const size_t nact = kmb_block_activation_floats(&c, 1);
    float* act = (float*)workspace(WS_BLK_WBF + 3, nact * sizeof(float));
    if (!zeros || !act) { set_error("workspace allocation failed"); return; }
    cudaMemsetAsync(zeros, 0, (size_t)NR * sizeof(float) * 2, 0);
    KMBlockWeights w = {d_W_in, d_W_out, d_A_log, d_W_B, d_W_C, d_delta_proj, d_lambda_proj, zeros, zeros + NR, d_theta};
    if (kmb_block_forward(&c, &w, d_x, d_y, 1, act, nullptr)) return;
    const ActLayout a = act_layout(&c, 1);
    gather_proj<<<nb(L, 256), 256>>>(act + a.proj, L, (int)a.Rt, (int)c.R, d_u_raw, d_dt_raw, d_lambda_raw);
    const size_t f = sizeof(float);
    cudaMemcpyAsync(d_u, act + a.u, (size_t)L * c.R * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_dt, act + a.dt, (size_t)L * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_lambda, act + a.lam, (size_t)L * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_B_exp, act + a.B, (size_t)L * NR * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_C_exp, act + a.C, (size_t)L * NR * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_h_store, act + a.h, (size_t)L * state * f, cudaMemcpyDeviceToDevice, 0);
    if (d_dt_exp) cudaMemcpyAsync(d_dt_exp, act + a.Bu, (size_t)L * state * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(d_y_scan, act + a.y, (size_t)L * c.R * f, cudaMemcpyDeviceToDevice, 0);
    if (d_y_proj) {  // y_proj = y - x
        cudaMemcpyAsync(d_y_proj, d_y, (size_t)L * dim * f, cudaMemcpyDeviceToDevice, 0);
        sub_inplace<<<nb((long long)L * dim, 256), 256>>>(d_y_proj, d_x, (long long)L * dim);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) set_cuda_error("cuda_block_forward", e);
}

extern "C" void cuda_block_backward(void* cublas, const float* d_W_in, const float* d_W_out, const float* d_A_log,
                                    const float* d_W_B, const float* d_W_C, const float* d_delta_proj,
                                    const float* d_theta, const float* d_lambda_proj, const float* d_x,
                                    const float* d_u_raw, const float* d_u, const float* d_dt_raw, const float* d_dt,
                                    const float* d_B_exp, const float* d_C_exp, const float* d_dt_exp,
                                    const float* d_h_store, const float* d_y_scan, const float* d_lambda,
                                    const float* d_dy, float* d_dW_in, float* d_dW_out, float* d_dA_log,
                                    float* d_dW_B, float* d_dW_C, float* d_ddelta_proj, float* d_g_theta,
                                    float* d_g_lambda_proj, float* d_dx, float* d_dy_scan, float* d_du,
                                    float* d_du_raw, float* d_ddt, float* d_ddt_raw, float* d_dB_scan,
                                    float* d_dC_scan, float* d_ddt_scan, float* d_dA_tmp, float* d_dlambda,
                                    float* d_dlambda_raw, int L, int state, int dim, int R, int spatial_ndims,
                                    const long* spatial_dims) {
    (void)cublas; (void)d_dy_scan; (void)d_du; (void)d_du_raw; (void)d_ddt; (void)d_ddt_raw; (void)d_dB_scan;
    (void)d_dC_scan; (void)d_ddt_scan; (void)d_dA_tmp; (void)d_dlambda; (void)d_dlambda_raw;
    clear_error();
    KMBlockConfig c = ref_cfg(L, state, dim, R, spatial_ndims, spatial_dims);
    const long long NR = (long long)state * c.R;
    float* zeros = (float*)workspace(WS_BLK_WBF + 2, (size_t)NR * sizeof(float) * 2);
    const size_t nact = kmb_block_activation_floats(&c, 1);
    float* act = (float*)workspace(WS_BLK_WBF + 3, nact * sizeof(float));
    if (!zeros || !act) { set_error("workspace allocation failed"); return; }
    cudaMemsetAsync(zeros, 0, (size_t)NR * sizeof(float) * 2, 0);
    const ActLayout a = act_layout(&c, 1);
    // rebuild the packed activations: P columns from the raw buffers (B / C columns are only
    // copied for completeness; the backward reads u_raw, dt_raw from P and the rest from the arrays)
    // lambda_raw is not passed to the reference backward; P's lambda column is unused by the backward.
    scatter_proj<<<nb(L, 256), 256>>>(act + a.proj, L, (int)a.Rt, (int)c.R, (int)NR, d_u_raw, d_dt_raw, nullptr,
                                      d_B_exp, d_C_exp);
    const size_t f = sizeof(float);
    cudaMemcpyAsync(act + a.u, d_u, (size_t)L * c.R * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(act + a.dt, d_dt, (size_t)L * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(act + a.lam, d_lambda, (size_t)L * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(act + a.B, d_B_exp, (size_t)L * NR * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(act + a.C, d_C_exp, (size_t)L * NR * f, cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(act + a.h, d_h_store, (size_t)L * state * f, cudaMemcpyDeviceToDevice, 0);
    if (d_dt_exp)
        cudaMemcpyAsync(act + a.Bu, d_dt_exp, (size_t)L * state * f, cudaMemcpyDeviceToDevice, 0);
    else
        rebuild_bu<<<nb((long long)L * state, 256), 256>>>(d_B_exp, d_u, L, state, (int)c.R, act + a.Bu);
    cudaMemcpyAsync(act + a.y, d_y_scan, (size_t)L * c.R * f, cudaMemcpyDeviceToDevice, 0);
    KMBlockWeights w = {d_W_in, d_W_out, d_A_log, d_W_B, d_W_C, d_delta_proj, d_lambda_proj, zeros, zeros + NR, d_theta};
    KMBlockGrads g = {d_dW_in, d_dW_out, d_dA_log, d_dW_B, d_dW_C, d_ddelta_proj, d_g_lambda_proj, nullptr, nullptr,
                      d_g_theta};
    kmb_block_backward(&c, &w, d_x, d_dy, d_dx, &g, 1, act, nullptr);
}
