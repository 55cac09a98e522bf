// proj_tc.cu -- the bf16 block projection on the sm_100a tensor cores (tcgen05),
// with the block's input epilogue fused in.
//
// Q[row, c] = sum_k X[row, k] Wtc[c, k]   (X [BL, dim] bf16, Wtc [Rt, dim] bf16,
// both K-major), with the projection rows in the order Wtc = [W_B; W_C; W_in;
// delta_proj; lambda_proj] so that 16-column accumulator chunks map onto whole
// 32-byte pieces of B and C rows (N R % 16 == 0).  Then per column (reference
// project_controller_full, src/mamba_block.c:106-125): B = Q + b_B and C = Q +
// b_C, u = silu(Q), dt = clamp(softplus(Q)), lambda = sigmoid(Q).  u, dt,
// lambda, B, C are written as bf16 straight from the accumulator (B and C as
// 16-byte vectors); the fp32 pre-activations of u, dt, lambda are also kept in
// the block's P layout (row stride Rt, columns 0 .. R+1), which is all the
// backward epilogue reads of P.
//
// One CTA per 128-row tile of X and up to 256 columns of Wcat (grid.y covers
// more; two CTAs per SM): warp 0 issues the TMA loads (128B-swizzled K-major
// tiles, 64 K-elements per stage, a ring of S stages), warp 1 owns the TMEM
// accumulator (128 lanes x up to 256 fp32 columns) and issues tcgen05.mma
// (M = 128, N <= 256, K = 16 per instruction), warps 2-5 read TMEM rows back with
// tcgen05.ld and run the epilogue.  Every wait is bounded; on a timeout the
// kernel records a status, drains its copies and still frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include "kmb_common.cuh"
#include "kmb_sync.cuh"

namespace kmb {

// D[row, c] = sum_k A[row, k] Bm[c, k] over K, for N output columns, then one of
// two epilogues: EPI 0 = the block's input projection (above), EPI 1 = the
// input gradient of the block, dx = bf16(dout + D) (row stride N).
struct ProjTCDesc {
    long long BL;
    int K, N;                         // reduction length, output columns
    int R, NR, Rt, ncols_max;         // ncols_max: columns one CTA covers (<= 512, multiple of 16)
    const __nv_bfloat16* dout;        // EPI 1
    __nv_bfloat16* dx;
    int stages, stage_bytes, x_bytes;
    float dt_min, dt_max;
    const float *bB, *bC;
    float* P;                         // fp32 pre-activations, [BL, Rt] (columns < R + 2 written)
    __nv_bfloat16 *u, *dt, *lam, *B, *C;
    int* status;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((unsigned long long)map), "r"(bar), "r"(c0), "r"(c1) : "memory");
}

// K-major, 128-byte-swizzled operand tile: rows of 64 bf16 (128 B), 8-row groups
// 1024 B apart; start must be 1024-byte aligned (+ 32 B per K step of 16).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    const uint64_t lo = (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16);   // start, LBO = 16 B (unused)
    const uint64_t hi = (uint64_t)(1024 >> 4) | ((uint64_t)1 << 14) | ((uint64_t)2 << 29);  // SBO, version 1, SW128
    return lo | (hi << 32);
}
// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, M = 128
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)acc) : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive TMEM columns of this warp's 32 lanes, waited for inside the same asm
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, "
        "%36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, "
        "%57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = __uint_as_float(r[i]);
}

constexpr int PTC_THREADS = 192;
constexpr int PTC_WROWS = 16;   // rows of Wcat per TMA box

template <int EPI>
__global__ void __launch_bounds__(PTC_THREADS, 1)
proj_fwd_tc(const __grid_constant__ ProjTCDesc d, const __grid_constant__ CUtensorMap mX,
            const __grid_constant__ CUtensorMap mW) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int S = d.stages;
    uint64_t* full = (uint64_t*)(smem + (size_t)S * d.stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* done = empty + S;
    uint32_t* tmem_slot = (uint32_t*)(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long m0 = (long long)blockIdx.x * 128;
    const int n0 = blockIdx.y * d.ncols_max;
    const int ncols = min(d.ncols_max, ((d.N + 15) & ~15) - n0);   // multiple of 16
    const int nch0 = min(ncols, 256), nch1 = ncols - nch0;
    const int nkb = (d.K + 63) / 64;
    const int tcols = ncols <= 32 ? 32 : ncols <= 64 ? 64 : ncols <= 128 ? 128 : ncols <= 256 ? 256 : 512;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), 1);
        }
        mbar_init(smem_u32(done), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            const unsigned wbytes = (unsigned)ncols * 128;
            int issued = 0;
            for (int kb = 0; kb < nkb && ok; kb++) {
                const int s = kb % S;
                if (kb >= S && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(((kb / S) - 1) & 1))) {
                    set_status(d.status, KMB_ERR_TIMEOUT_EMPTY);
                    ok = false;
                    break;
                }
                unsigned char* st = smem + (size_t)s * d.stage_bytes;
                const uint32_t fb = smem_u32(&full[s]);
                mbar_expect_tx(fb, (unsigned)d.x_bytes + wbytes);
                tma_load_2d(smem_u32(st), &mX, fb, kb * 64, (int)m0);
                for (int r = 0; r < ncols; r += PTC_WROWS)
                    tma_load_2d(smem_u32(st + d.x_bytes + r * 128), &mW, fb, kb * 64, n0 + r);
                issued = kb + 1;
            }
            // copies still in flight must land before the CTA can leave
            for (int kb = (issued > S ? issued - S : 0); kb < issued; kb++)
                mbar_wait(smem_u32(&full[kb % S]), (uint32_t)((kb / S) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id0 = idesc_bf16(nch0), id1 = nch1 > 0 ? idesc_bf16(nch1) : 0u;
            for (int kb = 0; kb < nkb; kb++) {
                const int s = kb % S;
                if (!mbar_wait(smem_u32(&full[s]), (uint32_t)((kb / S) & 1))) {
                    set_status(d.status, KMB_ERR_TIMEOUT_FULL);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t xa = smem_u32(smem + (size_t)s * d.stage_bytes);
                const uint32_t wa = xa + d.x_bytes;
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const bool acc = kb > 0 || ks > 0;
                    umma_bf16(tmem, sw128_desc(xa + ks * 32), sw128_desc(wa + ks * 32), id0, acc);
                    if (nch1 > 0)
                        umma_bf16(tmem + 256, sw128_desc(xa + ks * 32), sw128_desc(wa + 256 * 128 + ks * 32), id1, acc);
                }
                umma_commit(smem_u32(&empty[s]));   // the stage is free once these MMAs have read it
            }
            umma_commit(smem_u32(done));            // accumulator complete (or as far as it got)
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = rows of the tile
        const int q = warp & 3;
        const long long row = m0 + q * 32 + lane;
        const bool got = mbar_wait(smem_u32(done), 0);
        if (!got) set_status(d.status, KMB_ERR_TIMEOUT_Y);
        tc_fence_after();
        const int R = d.R, NR = d.NR, Rt = d.Rt;
        // one 16-column chunk of this row: v = the accumulator, dv = the dout chunk (EPI 1)
        auto chunk = [&](int c, const float* v, const uint4* dv) {
            const int col = n0 + c;
            if constexpr (EPI == 1) {
                // dx = bf16(dout + D): 16 columns, two 16-byte stores (dx may alias dout: read before)
                const long long o = row * d.N + col;
                uint4 pk[2] = {dv[0], dv[1]};
                __nv_bfloat16* e = (__nv_bfloat16*)pk;
#pragma unroll
                for (int j = 0; j < 16; j++) e[j] = __float2bfloat16_rn(__bfloat162float(e[j]) + v[j]);
                ((uint4*)(d.dx + o))[0] = pk[0];
                ((uint4*)(d.dx + o))[1] = pk[1];
                return;
            }
            if (col < 2 * NR) {
                // 16 columns of B or C: bias, round, two 16-byte stores
                const bool isB = col < NR;
                const int jj = isB ? col : col - NR;
                const float* bias = (isB ? d.bB : d.bC) + jj;
                __nv_bfloat16* dst = (isB ? d.B : d.C) + row * NR + jj;
                uint4 pk[2];
                __nv_bfloat16* e = (__nv_bfloat16*)pk;
#pragma unroll
                for (int j = 0; j < 16; j++) e[j] = __float2bfloat16_rn(v[j] + bias[j]);
                ((uint4*)dst)[0] = pk[0];
                ((uint4*)dst)[1] = pk[1];
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int k = col + j - 2 * NR;  // 0 .. R-1: u, R: dt, R+1: lambda
                    if (k > R + 1) break;
                    const float z = v[j];
                    d.P[row * Rt + k] = z;
                    if (k < R) {
                        d.u[row * R + k] = __float2bfloat16_rn(z / (1.0f + expf(-z)));
                    } else if (k == R) {
                        float t = logf(1.0f + expf(z));
                        t = fminf(fmaxf(t, d.dt_min), d.dt_max);
                        d.dt[row] = __float2bfloat16_rn(t);
                    } else {
                        d.lam[row] = __float2bfloat16_rn(1.0f / (1.0f + expf(-z)));
                    }
                }
            }
        };
        const bool live = got && row < d.BL;
        int c = 0;
        // 64 columns at a time: the row's dout loads (EPI 1) and one TMEM load in flight together
        for (; c + 64 <= ncols; c += 64) {
            uint4 dv[8];
            if (EPI == 1 && live) {
                const uint4* src = (const uint4*)(d.dout + row * d.N + n0 + c);
#pragma unroll
                for (int i = 0; i < 8; i++) dv[i] = src[i];
            }
            float v[64];
            tmem_ld64(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
            if (!live) continue;
#pragma unroll
            for (int i = 0; i < 4; i++) chunk(c + 16 * i, v + 16 * i, dv + 2 * i);
        }
        for (; c < ncols; c += 16) {
            uint4 dv[2];
            if (EPI == 1 && live) {
                const uint4* src = (const uint4*)(d.dout + row * d.N + n0 + c);
                dv[0] = src[0];
                dv[1] = src[1];
            }
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
            if (!live) continue;
            chunk(c, v, dv);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

// Wtc[Rt, dim] bf16 = [W_B; W_C; W_in; delta_proj; lambda_proj]
__global__ void pack_wtc(const float* __restrict__ Win, const float* __restrict__ dp, const float* __restrict__ lp,
                         const float* __restrict__ WB, const float* __restrict__ WC, int R, int NR, int dim,
                         __nv_bfloat16* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long Rt = R + 2 + 2LL * NR;
    if (i >= Rt * dim) return;
    const int row = (int)(i / dim), col = (int)(i - (long long)row * dim);
    float v;
    if (row < NR) v = WB[(long long)row * dim + col];
    else if (row < 2 * NR) v = WC[(long long)(row - NR) * dim + col];
    else if (row < 2 * NR + R) v = Win[(long long)(row - 2 * NR) * dim + col];
    else if (row == 2 * NR + R) v = dp[col];
    else v = lp[col];
    out[i] = __float2bfloat16_rn(v);
}

bool tmap_encode_ex(CUtensorMap* m, const void* base, int dtype, int rank, const unsigned long long* dims,
                    const unsigned long long* strides_bytes, const unsigned* box, int swizzle);

// Returns cudaErrorNotSupported when the shapes do not fit this kernel.
// Wt[dim, ldp] bf16 = Wcat^T (Wcat = [W_in; delta_proj; lambda_proj; W_B; W_C], [Rt, dim]); columns
// Rt .. ldp-1 are zero
__global__ void pack_wcat_t(const float* __restrict__ Win, const float* __restrict__ dp, const float* __restrict__ lp,
                            const float* __restrict__ WB, const float* __restrict__ WC, int R, int NR, int dim,
                            int ldp, __nv_bfloat16* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)dim * ldp) return;
    const int n = (int)(i / ldp), c = (int)(i - (long long)n * ldp);
    float v = 0.0f;
    if (c < R) v = Win[(long long)c * dim + n];
    else if (c == R) v = dp[n];
    else if (c == R + 1) v = lp[n];
    else if (c < R + 2 + NR) v = WB[(long long)(c - R - 2) * dim + n];
    else if (c < R + 2 + 2 * NR) v = WC[(long long)(c - R - 2 - NR) * dim + n];
    out[i] = __float2bfloat16_rn(v);
}

cudaError_t launch_pack_wcat_t(const float* Win, const float* dp, const float* lp, const float* WB, const float* WC,
                               int R, int NR, int dim, int ldp, __nv_bfloat16* out, cudaStream_t st) {
    pack_wcat_t<<<(unsigned)(((long long)dim * ldp + 255) / 256), 256, 0, st>>>(Win, dp, lp, WB, WC, R, NR, dim, ldp,
                                                                               out);
    return cudaGetLastError();
}

// Stage sizing, tensor maps and launch shared by both epilogues.  A [M, K] and
// Bm [N, K] are bf16, K-major, with row strides lda / ldb elements.
template <int EPI>
static cudaError_t tc_launch(ProjTCDesc& d, const __nv_bfloat16* A, int lda, const __nv_bfloat16* Bm, int ldb,
                             cudaStream_t st) {
    if (((uintptr_t)A & 15) || ((uintptr_t)Bm & 15) || (lda % 8) || (ldb % 8) || d.BL < 1 || d.K < 1 || d.N < 16)
        return cudaErrorNotSupported;
    const int npad = (d.N + 15) & ~15;
    // 256-column ranges and <= 110 KB of stages: two CTAs (and two 256-column TMEM
    // accumulators) per SM, so one tile's epilogue overlaps another's loads and MMAs
    d.ncols_max = npad <= 256 ? npad : 256;
    d.x_bytes = 128 * 128;
    d.stage_bytes = d.x_bytes + d.ncols_max * 128;
    d.stages = (110 * 1024) / d.stage_bytes;
    if (d.stages > 4) d.stages = 4;
    if (d.stages < 2) return cudaErrorNotSupported;
    CUtensorMap mA, mB;
    {
        const unsigned long long dims[2] = {(unsigned long long)d.K, (unsigned long long)d.BL};
        const unsigned long long str[1] = {(unsigned long long)lda * 2};
        const unsigned box[2] = {64, 128};
        if (!tmap_encode_ex(&mA, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorNotSupported;
    }
    {
        const unsigned long long dims[2] = {(unsigned long long)d.K, (unsigned long long)d.N};
        const unsigned long long str[1] = {(unsigned long long)ldb * 2};
        const unsigned box[2] = {64, PTC_WROWS};
        if (!tmap_encode_ex(&mB, Bm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorNotSupported;
    }
    const int smem = 1024 + d.stages * d.stage_bytes + (2 * d.stages + 1) * 8 + 16;
    cudaError_t e = cudaFuncSetAttribute(proj_fwd_tc<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((d.BL + 127) / 128), (unsigned)((npad + d.ncols_max - 1) / d.ncols_max));
    proj_fwd_tc<EPI><<<grid, PTC_THREADS, smem, st>>>(d, mA, mB);
    return cudaGetLastError();
}

// dx[BL, dim] = bf16(dout + dP Wcat) for the bf16 block backward.  dP is [BL, ldp]
// bf16 with zero columns Rt .. ldp-1; Wt is bf16 scratch of dim x ldp.
cudaError_t launch_dx_tc(const __nv_bfloat16* dP, int ldp, const float* Win, const float* dp, const float* lp,
                         const float* WB, const float* WC, __nv_bfloat16* Wt, long long BL, int dim, int R, int NR,
                         const __nv_bfloat16* dout, __nv_bfloat16* dx, int* status, cudaStream_t st) {
    if (dim % 16 != 0 || ((uintptr_t)dout & 15) || ((uintptr_t)dx & 15) || ((uintptr_t)Wt & 15))
        return cudaErrorNotSupported;
    ProjTCDesc d{};
    d.BL = BL; d.K = ldp; d.N = dim; d.R = R; d.NR = NR; d.Rt = R + 2 + 2 * NR;
    d.dout = dout; d.dx = dx; d.status = status;
    pack_wcat_t<<<(unsigned)(((long long)dim * ldp + 255) / 256), 256, 0, st>>>(Win, dp, lp, WB, WC, R, NR, dim, ldp,
                                                                               Wt);
    return tc_launch<1>(d, dP, ldp, Wt, ldp, st);
}

// W: bf16 scratch of Rt x dim for the reordered weights.
cudaError_t launch_proj_fwd_tc(const __nv_bfloat16* X, const float* Win, const float* dp, const float* lp,
                               const float* WB, const float* WC, __nv_bfloat16* W, long long BL, int dim, int R,
                               int NR, float dt_min, float dt_max, const float* bB, const float* bC, float* P,
                               __nv_bfloat16* u, __nv_bfloat16* dt, __nv_bfloat16* lam, __nv_bfloat16* B,
                               __nv_bfloat16* C, int* status, cudaStream_t st) {
    const int Rt = R + 2 + 2 * NR;
    if (NR % 16 != 0 || R + 2 > 16 || ((uintptr_t)X & 15) || ((uintptr_t)W & 15) ||
        ((uintptr_t)B & 15) || ((uintptr_t)C & 15) || BL < 1)
        return cudaErrorNotSupported;
    pack_wtc<<<(unsigned)(((long long)Rt * dim + 255) / 256), 256, 0, st>>>(Win, dp, lp, WB, WC, R, NR, dim, W);
    ProjTCDesc d{};
    d.BL = BL; d.K = dim; d.N = Rt; d.R = R; d.NR = NR; d.Rt = Rt;
    d.dt_min = dt_min; d.dt_max = dt_max; d.bB = bB; d.bC = bC; d.P = P;
    d.u = u; d.dt = dt; d.lam = lam; d.B = B; d.C = C; d.status = status;
    return tc_launch<0>(d, X, dim, W, dim, st);
}

}  // namespace kmb
