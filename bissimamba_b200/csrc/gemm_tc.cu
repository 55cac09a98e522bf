// gemm_tc.cu -- the block and model GEMMs on the sm_100a tensor cores
// (tcgen05), in place of library GEMMs:
//
//   D[m, n] (+)= sum_k A[m, k] B[n, k]
//
// Operands are K-major ([rows, K] row-major) or, for 16-bit kinds, MN-major
// ([K, rows] row-major: the transposed product A^T B of two row-major
// matrices needs no transposition pass).  Kinds, by the pieces each operand
// is given as:
//   KIND_BF16    one bf16 piece, kind::f16 MMAs;
//   KIND_TF32X3  fp32 at fp32 accuracy, two fp32 pieces hi = rna_tf32(x) and
//                lo = rna_tf32(x - hi): hi_a lo_b + lo_a hi_b + hi_a hi_b
//                (kind::tf32), a relative error of about 2^-22 per product;
//   KIND_BF16X6  fp32 at fp32 accuracy, three bf16 pieces x = b0 + b1 + b2
//                (each the bf16 rounding of what the previous ones leave; the
//                remainder is below 2^-26 |x|), the six products of order
//                <= 2, smallest first, kind::f16 (the split-bf16 emulation of
//                an fp32 GEMM: Henry, Tang, Heinecke, "Leveraging the bfloat16
//                artificial intelligence datatype for higher-precision
//                computations", ARITH 2019);
//   KIND_BF16X9  the same with all nine products.
// One CTA per 128-row tile of A and a column tile of B; grid.x walks the
// column tiles, so the CTAs that share an A tile run together and read it
// from L2.  Warp 0 issues TMA loads into a ring of stages, warp 1 allocates
// TMEM and issues the MMAs, warps 2-9 read the accumulator back (tcgen05.ld)
// and store through shared memory.  bf16: 128-byte swizzled rows (64 K per
// stage), up to 256 columns, two CTAs per SM.  fp32 kinds: 64-byte swizzled
// rows (32 K per stage), up to 192 columns, three stages of the operand
// pieces, one CTA per SM.
// The fp32 kinds do not let one TMEM accumulator run over all of K: the
// tensor core's accumulation drifts with the number of products it adds (its
// error grows about as sqrt(K) relative to sum |a b|, where an fp32 FMA loop's
// stays flat).  The leading product (a0 b0, or hi hi) accumulates in one TMEM
// buffer for `kflush` MMA K steps (16 bf16 or 8 tf32 K each) at a time, after
// which the epilogue warps add it into an fp32 running sum in registers; the
// smaller products, 2^-8 (2^-11) of its size and smaller, accumulate over all
// of K in a second buffer whose drift stays below fp32 rounding, added once at
// the end.
// Split-K: grid.z cuts K into chunks; each split writes its own partial
// (EPI_STORE at D + split * split_stride), summed later in a fixed order.
// EPI_ADD adds the accumulator into D (one split).  Every wait is bounded; on a
// timeout the kernel records a status, drains its copies and frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include "kmb_common.cuh"
#include "kmb_sync.cuh"
#include "kmb_gemm.cuh"

namespace kmb {

bool tmap_encode_ex(CUtensorMap* m, const void* base, int dtype, int rank, const unsigned long long* dims,
                    const unsigned long long* strides_bytes, const unsigned* box, int swizzle);

enum { KIND_BF16 = 0, KIND_TF32X3 = 1, KIND_BF16X6 = 2, KIND_BF16X9 = 3 };
enum { EPI_STORE = 0, EPI_ADD = 1 };

struct GemmTCDesc {
    long long M, N, K;
    long long kchunk;          // K per split (a multiple of the stage depth)
    int ncols_max;             // columns per CTA (<= 256)
    int stages, a_bytes, b_bytes, stage_bytes;
    int kflush;                // fp32 kinds: MMA K steps per TMEM buffer (1, 2 or 4)
    int tbuf;                  // fp32 kinds: TMEM columns per buffer (128 or 192)
    float* D;
    long long ldd;
    long long split_stride;    // elements between the splits' partial outputs
    int* status;
};

namespace {

template <int KIND> struct KindTraits;
template <> struct KindTraits<KIND_BF16> { static constexpr int NP = 1, ESZ = 2, NPROD = 1; };
template <> struct KindTraits<KIND_TF32X3> { static constexpr int NP = 2, ESZ = 4, NPROD = 3; };
template <> struct KindTraits<KIND_BF16X6> { static constexpr int NP = 3, ESZ = 2, NPROD = 6; };
template <> struct KindTraits<KIND_BF16X9> { static constexpr int NP = 3, ESZ = 2, NPROD = 9; };

// piece pairs (a, b), smallest products first, the leading product last
__device__ __forceinline__ void prod_pair(int kind, int i, int& pa, int& pb) {
    if (kind == KIND_BF16) { pa = 0; pb = 0; return; }
    if (kind == KIND_TF32X3) {
        const int a[3] = {1, 0, 0}, b[3] = {0, 1, 0};
        pa = a[i]; pb = b[i];
        return;
    }
    // x9: (2,2) (2,1) (1,2) then the x6 list (2,0) (1,1) (0,2) (1,0) (0,1) (0,0)
    const int a[9] = {2, 2, 1, 2, 1, 0, 1, 0, 0}, b[9] = {2, 1, 2, 0, 1, 2, 0, 1, 0};
    const int off = kind == KIND_BF16X9 ? 0 : 3;
    pa = a[off + i]; pb = b[off + i];
}

__device__ __forceinline__ void g_tma_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((unsigned long long)map), "r"(bar), "r"(c0), "r"(c1) : "memory");
}
// Swizzled shared-memory matrix descriptor (sm_100 form: bit 46 set; layout type in bits 61-63: 2 = 128-byte,
// 4 = 64-byte swizzle).  K-major: 8-row groups SBO apart (8 rows of the swizzle width), LBO unused.  MN-major:
// LBO = bytes between MN blocks (one TMA box apart), SBO = bytes between 8-row K groups.
__device__ __forceinline__ uint64_t g_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t mode) {
    const uint64_t lo = (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16);
    const uint64_t hi = (uint64_t)((sbo >> 4) & 0x3FFF) | ((uint64_t)1 << 14) | ((uint64_t)mode << 29);
    return lo | (hi << 32);
}
// instruction descriptor: fp32 accumulator, A / B format (1 = bf16, 2 = tf32), major-ness (bit 15 A,
// bit 16 B: 1 = MN-major), N, M = 128
__device__ __forceinline__ uint32_t g_idesc(int fmt, int n, bool mn) {
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | (mn ? (3u << 15) : 0u) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
template <int KIND>
__device__ __forceinline__ void g_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, bool acc) {
    if constexpr (KIND == KIND_TF32X3)
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(d), "l"(a), "l"(b), "r"(id), "r"((uint32_t)acc) : "memory");
    else
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(d), "l"(a), "l"(b), "r"(id), "r"((uint32_t)acc) : "memory");
}
__device__ __forceinline__ void g_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void g_ld16(uint32_t taddr, float (&v)[16]) {
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
__device__ __forceinline__ void g_ld64(uint32_t taddr, float* v) {
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

// 32 consecutive TMEM columns of this warp's 32 lanes, waited for inside the same asm
__device__ __forceinline__ void g_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// The epilogue's 256 threads (warps 2-9: lane quarter q = warp % 4 of TMEM, column group hh) write the CTA's
// fp32 block through shared memory so that global stores are whole 128-byte rows: a row-major tile of TW
// columns with a TW + 1 float stride (conflict-free both ways; bf16 passes 128 columns at a time, the fp32
// kinds all of their <= 192 columns at once).
constexpr int EPI_WARPS = 8;
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
template <int EPI, int NV, int TW>
__device__ __forceinline__ void epi_flush(float* tile, int q, int hh, const float* vals, int nv, int cb,
                                          int cols_here, float* D, long long ldd, long long m0, long long M,
                                          long long col0, long long N, int lane, bool write) {
    // every epilogue thread reaches both barriers; `write` only gates the stores.  This thread holds
    // tile columns cb .. cb + nv - 1 of its row (nv <= NV).
    constexpr int LD = TW + 1;
    const int rl = q * 32 + lane;
#pragma unroll
    for (int c = 0; c < NV; c++)
        if (c < nv && cb + c < cols_here) tile[rl * LD + cb + c] = vals[c];
    epi_bar();
    // epilogue warp e = hh * 4 + q writes rows 16 e .. 16 e + 15, lanes along the columns; EPI_ADD loads
    // two rows' worth of D before it stores any, so the loads overlap
    const int e = hh * 4 + q;
    constexpr int KW = TW / 32;
    if (write) {
        for (int i0 = 0; i0 < 16; i0 += 2) {
            float g[2][KW];
            if (EPI == EPI_ADD) {
#pragma unroll
                for (int i = 0; i < 2; i++)
#pragma unroll
                    for (int k = 0; k < KW; k++) {
                        const int r = e * 16 + i0 + i, c = lane + 32 * k;
                        const long long row = m0 + r, col = col0 + c;
                        g[i][k] = (row < M && c < cols_here && col < N) ? D[row * ldd + col] : 0.0f;
                    }
            }
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int k = 0; k < KW; k++) {
                    const int r = e * 16 + i0 + i, c = lane + 32 * k;
                    const long long row = m0 + r, col = col0 + c;
                    if (row < M && c < cols_here && col < N) {
                        const float t = tile[r * LD + c];
                        D[row * ldd + col] = EPI == EPI_ADD ? g[i][k] + t : t;
                    }
                }
        }
    }
    epi_bar();
}

constexpr int GT_THREADS = 64 + 32 * EPI_WARPS;   // TMA warp, MMA warp, 8 epilogue warps

// Geometry of one instantiation.  bf16: 128-byte swizzle, 64 K per stage, up to 256 columns, one TMEM
// accumulator.  fp32 kinds: 64-byte swizzle, 32 K per stage (so three stages of three pieces fit with
// 256-column tiles), two TMEM buffers of up to 256 columns each.
template <int KIND, bool MN>
struct GtGeom {
    static constexpr bool FL = KIND != KIND_BF16;
    static constexpr int ESZ = KindTraits<KIND>::ESZ;
    static constexpr int ROWB = FL ? 64 : 128;                 // bytes of one swizzled row
    static constexpr uint32_t MODE = FL ? 4u : 2u;             // descriptor layout type
    static constexpr int MNB = ROWB / 2;                       // MN-major: elements per box row
    static constexpr int KS = MN ? ROWB / 2 : ROWB / ESZ;      // K per stage
    static constexpr int KSTEPS = MN ? KS / 16 : ROWB / 32;    // MMAs (K steps) per stage and product
    static constexpr int BOXB = ROWB * KS;                     // MN-major: bytes of one box (MNB x KS)
    static constexpr uint32_t SBO = 8 * ROWB;
};

// Stage layout: A pieces 0..NP-1 (a_bytes each), then B pieces (b_bytes each).
// K-major: one TMA box per piece and operand ([128 or ncols rows] x ROWB).
// MN-major: boxes of MNB elements x KS K rows, side by side.
template <int KIND, int EPI, bool MN>
__global__ void __launch_bounds__(GT_THREADS, KIND == KIND_BF16 ? 2 : 1)
gemm_tc_kernel(const __grid_constant__ GemmTCDesc d, const __grid_constant__ CUtensorMap mA0,
               const __grid_constant__ CUtensorMap mA1, const __grid_constant__ CUtensorMap mA2,
               const __grid_constant__ CUtensorMap mB0, const __grid_constant__ CUtensorMap mB1,
               const __grid_constant__ CUtensorMap mB2) {
    using TR = KindTraits<KIND>;
    using GG = GtGeom<KIND, MN>;
    constexpr int NP = TR::NP;
    constexpr int KS = GG::KS, KSTEPS = GG::KSTEPS, MNB = GG::MNB, BOXB = GG::BOXB;
    constexpr bool FL = GG::FL;   // accumulator flush every kflush K steps
    extern __shared__ __align__(1024) unsigned char g_smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)g_smem_raw + 1023) & ~(uintptr_t)1023);
    const int S = d.stages;
    uint64_t* full = (uint64_t*)(smem + (size_t)S * d.stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* done = empty + S;
    uint64_t* tfull = done + 1;     // FL: TMEM buffer b holds a finished unit
    uint64_t* tempty = done + 3;    // FL: the epilogue has read TMEM buffer b
    uint32_t* tmem_slot = (uint32_t*)(done + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long n0 = (long long)blockIdx.x * d.ncols_max;
    const long long m0 = (long long)blockIdx.y * 128;
    const int ncols = (int)min((long long)d.ncols_max, ((d.N + 15) & ~15LL) - n0);   // multiple of 16
    const long long k0 = (long long)blockIdx.z * d.kchunk;
    const long long k1 = min(d.K, k0 + d.kchunk);
    const int nkb = k1 > k0 ? (int)((k1 - k0 + KS - 1) / KS) : 0;
    const int TB = d.tbuf;          // FL: columns between the two TMEM buffers (128 or 192)
    // (TMEM allocations are powers of two: two 192-column buffers take 512 columns)
    const int tcols = FL ? (TB <= 128 ? 256 : 512) : ncols <= 32 ? 32 : ncols <= 64 ? 64 : ncols <= 128 ? 128 : 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), 1);
        }
        mbar_init(smem_u32(done), 1);
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_u32(&tfull[b]), 1);
            mbar_init(smem_u32(&tempty[b]), EPI_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int total = nkb * KSTEPS;                    // MMA K steps of this CTA
    const int kf = FL ? d.kflush : 1;
    const int nunits = FL ? (total + kf - 1) / kf : 0;

    if (warp == 0) {
        if (lane == 0) {
            // rows past M or N and K past the end arrive zero-filled and count in the transaction bytes
            const int nbb = MN ? (ncols + MNB - 1) / MNB : 1;   // MN-major B boxes of this CTA
            const unsigned bytes = (unsigned)(NP * (d.a_bytes + (MN ? nbb * BOXB : d.b_bytes)));
            int issued = 0;
            for (int kb = 0; kb < nkb; kb++) {
                const int s = kb % S;
                if (kb >= S && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(((kb / S) - 1) & 1))) {
                    set_status(d.status, KMB_ERR_TIMEOUT_EMPTY);
                    break;
                }
                unsigned char* st = smem + (size_t)s * d.stage_bytes;
                const uint32_t fb = smem_u32(&full[s]);
                const int kc = (int)(k0 + (long long)kb * KS);
                mbar_expect_tx(fb, bytes);
#pragma unroll
                for (int p = 0; p < NP; p++) {
                    const CUtensorMap* mpa = p == 0 ? &mA0 : p == 1 ? &mA1 : &mA2;
                    const CUtensorMap* mpb = p == 0 ? &mB0 : p == 1 ? &mB1 : &mB2;
                    unsigned char* sa = st + p * d.a_bytes;
                    unsigned char* sb = st + NP * d.a_bytes + p * d.b_bytes;
                    if (MN) {
#pragma unroll
                        for (int i = 0; i < 128 / MNB; i++)
                            g_tma_2d(smem_u32(sa + i * BOXB), mpa, fb, (int)m0 + i * MNB, kc);
                        for (int bx = 0; bx < nbb; bx++)
                            g_tma_2d(smem_u32(sb + bx * BOXB), mpb, fb, (int)(n0 + MNB * bx), kc);
                    } else {
                        g_tma_2d(smem_u32(sa), mpa, fb, kc, (int)m0);
                        g_tma_2d(smem_u32(sb), mpb, fb, kc, (int)n0);
                    }
                }
                issued = kb + 1;
            }
            for (int kb = (issued > S ? issued - S : 0); kb < issued; kb++)
                mbar_wait(smem_u32(&full[kb % S]), (uint32_t)((kb / S) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const int fmt = KIND == KIND_TF32X3 ? 2 : 1;
            const uint32_t id = g_idesc(fmt, ncols, MN);
            const uint32_t lbo = MN ? (uint32_t)BOXB : 16u, sbo = GG::SBO;
            bool stop = false;
            for (int kb = 0; kb < nkb && !stop; kb++) {
                const int s = kb % S;
                if (!mbar_wait(smem_u32(&full[s]), (uint32_t)((kb / S) & 1))) {
                    set_status(d.status, KMB_ERR_TIMEOUT_FULL);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t st = smem_u32(smem + (size_t)s * d.stage_bytes);
#pragma unroll
                for (int ks = 0; ks < KSTEPS; ks++) {   // K-major: 32 bytes of K per MMA; MN-major: 16 K rows
                    const uint32_t o = MN ? ks * 16 * GG::ROWB : ks * 32;
                    const int g = kb * KSTEPS + ks, unit = g / kf;
                    const bool first = !FL ? (kb == 0 && ks == 0) : (g % kf == 0);
                    // FL: the leading product accumulates in the buffer at column 0, flushed every kflush K
                    // steps (wait until the epilogue has read the previous unit); the smaller products
                    // accumulate over all of K in the buffer at column TB
                    if (FL && first && unit >= 1 &&
                        !mbar_wait(smem_u32(&tempty[0]), (uint32_t)((unit - 1) & 1))) {
                        set_status(d.status, KMB_ERR_TIMEOUT_EMPTY);
                        stop = true;
                        break;
                    }
                    if (FL && first) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < TR::NPROD; i++) {
                        int pa, pb;
                        prod_pair(KIND, i, pa, pb);
                        const uint32_t a = st + pa * d.a_bytes + o;
                        const uint32_t b = st + NP * d.a_bytes + pb * d.b_bytes + o;
                        const bool lead = i == TR::NPROD - 1;
                        const uint32_t dt = (FL && !lead) ? tmem + (uint32_t)TB : tmem;
                        const bool acc = !FL ? (!first || i > 0) : lead ? !first : (g > 0 || i > 0);
                        g_mma<KIND>(dt, g_desc(a, lbo, sbo, GG::MODE), g_desc(b, lbo, sbo, GG::MODE), id, acc);
                    }
                    if (FL && (g % kf == kf - 1 || g == total - 1)) g_commit(smem_u32(&tfull[0]));
                }
                g_commit(smem_u32(&empty[s]));
            }
            g_commit(smem_u32(done));
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = rows of the tile; column group hh
        const int q = warp & 3, hh = (warp - 2) >> 2;
        float* dout = d.D + (long long)blockIdx.z * d.split_stride;
        if constexpr (FL) {
            // group hh (0, 1) holds columns hh * CG .. hh * CG + CG - 1 (CG = TB / 2 <= 96) as an fp32
            // running sum of the leading product's units, then adds the smaller products' accumulator
            const int CG = TB >> 1;
            float acc[96];
#pragma unroll
            for (int c = 0; c < 96; c++) acc[c] = 0.0f;
            bool ok = true;
            auto add_tmem = [&](uint32_t col0) {
                const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + col0 + (uint32_t)(hh * CG);
#pragma unroll
                for (int c = 0; c < 96; c += 16) {
                    if (c < CG && hh * CG + c < ncols) {
                        float v[16];
                        g_ld16(tb + (uint32_t)c, v);
#pragma unroll
                        for (int j = 0; j < 16; j++) acc[c + j] += v[j];
                    }
                }
            };
            for (int u = 0; u < nunits; u++) {
                if (!mbar_wait(smem_u32(&tfull[0]), (uint32_t)(u & 1))) {
                    set_status(d.status, KMB_ERR_TIMEOUT_Y);
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                add_tmem(0);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty[0]));
            }
            // the last commit covers every MMA; the stages are free for the store tile
            if (!mbar_wait(smem_u32(done), 0)) { set_status(d.status, KMB_ERR_TIMEOUT_Y); ok = false; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (ok && nkb > 0) add_tmem((uint32_t)TB);   // the smaller products, accumulated over all of K
            epi_flush<EPI, 96, 192>((float*)smem, q, hh, acc, CG, hh * CG, ncols, dout, d.ldd, m0, d.M, n0, d.N,
                                    lane, ok);
        } else {
            const bool got = mbar_wait(smem_u32(done), 0);
            if (!got) set_status(d.status, KMB_ERR_TIMEOUT_Y);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int h = 0; h < ncols; h += 128) {
                float v[64];
                if (h + hh * 64 < ncols && nkb > 0)
                    g_ld64(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h + hh * 64), v);
                else
#pragma unroll
                    for (int i = 0; i < 64; i++) v[i] = 0.0f;   // nkb == 0: an empty split stores zeros
                epi_flush<EPI, 64, 128>((float*)smem, q, hh, v, 64, hh * 64, min(128, ncols - h), dout, d.ldd, m0,
                                        d.M, n0 + h, d.N, lane, got);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

__device__ __forceinline__ float rna_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// hi = rna_tf32(x), lo = rna_tf32(x - hi) (x - hi is exact in fp32); four columns per thread
// (cols, ldx, ldo multiples of 4)
__global__ void split_tf32(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                           long long rows, int cols4, long long ldx, long long ldo) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols4) return;
    const long long r = i / cols4;
    const int c = (int)(i - r * cols4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
    const float e[4] = {v.x, v.y, v.z, v.w};
    float h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        h[k] = rna_tf32(e[k]);
        l[k] = rna_tf32(e[k] - h[k]);
    }
    *reinterpret_cast<float4*>(hi + r * ldo + c) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + r * ldo + c) = make_float4(l[0], l[1], l[2], l[3]);
}

// x = b0 + b1 + b2 (+ a remainder below 2^-26 |x|): each piece the bf16 rounding of what is left;
// four columns per thread (cols, ldx, ldo multiples of 4)
__global__ void split_bf16x3(const float* __restrict__ x, __nv_bfloat16* __restrict__ b0,
                             __nv_bfloat16* __restrict__ b1, __nv_bfloat16* __restrict__ b2, long long rows,
                             int cols4, long long ldx, long long ldo) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols4) return;
    const long long r = i / cols4;
    const int c = (int)(i - r * cols4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
    const float e[4] = {v.x, v.y, v.z, v.w};
    __align__(8) __nv_bfloat16 p0[4], p1[4], p2[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        p0[k] = __float2bfloat16_rn(e[k]);
        const float r1 = e[k] - __bfloat162float(p0[k]);
        p1[k] = __float2bfloat16_rn(r1);
        p2[k] = __float2bfloat16_rn(r1 - __bfloat162float(p1[k]));
    }
    *reinterpret_cast<uint2*>(b0 + r * ldo + c) = *reinterpret_cast<const uint2*>(p0);
    *reinterpret_cast<uint2*>(b1 + r * ldo + c) = *reinterpret_cast<const uint2*>(p1);
    *reinterpret_cast<uint2*>(b2 + r * ldo + c) = *reinterpret_cast<const uint2*>(p2);
}

// the same one element per thread, for any shape
__global__ void split_any(int kind, const float* __restrict__ x, void* o0, void* o1, void* o2, long long rows,
                          long long cols, long long ldx, long long ldo) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    const long long r = i / cols, c = i - r * cols;
    const float v = x[r * ldx + c];
    if (kind == KIND_TF32X3) {
        const float h = rna_tf32(v);
        ((float*)o0)[r * ldo + c] = h;
        ((float*)o1)[r * ldo + c] = rna_tf32(v - h);
    } else {
        const __nv_bfloat16 p0 = __float2bfloat16_rn(v);
        const float r1 = v - __bfloat162float(p0);
        const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
        ((__nv_bfloat16*)o0)[r * ldo + c] = p0;
        ((__nv_bfloat16*)o1)[r * ldo + c] = p1;
        ((__nv_bfloat16*)o2)[r * ldo + c] = __float2bfloat16_rn(r1 - __bfloat162float(p1));
    }
}

// out[c, r] = in[r, c]: in is R x Cn (row stride ldi), out Cn x R (row stride ldo); 32 x 32 tiles
template <typename T>
__global__ void transpose_2d(const T* __restrict__ in, T* __restrict__ out, long long R, long long Cn, long long ldi,
                             long long ldo) {
    __shared__ T t[32][33];
    const long long r0 = (long long)blockIdx.y * 32, c0 = (long long)blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const long long r = r0 + j, c = c0 + threadIdx.x;
        if (r < R && c < Cn) t[j][threadIdx.x] = in[r * ldi + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const long long c = c0 + j, r = r0 + threadIdx.x;   // out row c, column r
        if (r < R && c < Cn) out[c * ldo + r] = t[threadIdx.x][j];
    }
}

// out[i] (+)= sum_s part[s * stride + i], fixed order
__global__ void gt_reduce_splits(const float* __restrict__ part, float* __restrict__ out, long long n, int nsplit,
                                 long long stride, int accumulate, long long ldp, long long ldo, long long cols) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const long long r = i / cols, c = i - r * cols;
    float acc = 0.0f;
    for (int s = 0; s < nsplit; s++) acc += part[s * stride + r * ldp + c];
    float* o = out + r * ldo + c;
    *o = accumulate ? *o + acc : acc;
}

int g_kflush = 8;

int kind_pieces(int kind) { return kind == KIND_BF16 ? 1 : kind == KIND_TF32X3 ? 2 : 3; }


}  // namespace

// D = A B^T on the tensor cores (operands as in GemmOperand; MN-major only for
// the 16-bit kinds).  nsplit > 1 writes partials to D + s * split_stride.
// cudaErrorNotSupported when the shapes or alignments do not fit (rows of 16
// bytes: ld a multiple of 8 bf16 / 4 fp32, pieces 16-byte aligned).
cudaError_t gemm_tc(int kind, int epi, long long M, long long N, long long K, const GemmOperand& A,
                    const GemmOperand& B, float* D, long long ldd, int nsplit, long long split_stride, int* status,
                    cudaStream_t st) {
    const int NP = kind_pieces(kind);
    const int esz = kind == KIND_TF32X3 ? 4 : 2;
    const bool mn = A.mn_major != 0;
    if (M < 1 || N < 1 || K < 1 || nsplit < 1 || (A.mn_major != B.mn_major) || (mn && esz != 2) ||
        (A.ld * esz) % 16 || (B.ld * esz) % 16 || (epi == EPI_ADD && nsplit != 1) || M > 0x7fffffffLL ||
        N > 0x7fffffffLL || K > 0x7fffffffLL)
        return cudaErrorNotSupported;
    for (int p = 0; p < NP; p++)
        if (!A.p[p] || !B.p[p] || ((uintptr_t)A.p[p] & 15) || ((uintptr_t)B.p[p] & 15)) return cudaErrorNotSupported;
    // geometry (GtGeom): bf16 128-byte rows, the fp32 kinds 64-byte rows
    const bool fl = kind != KIND_BF16;
    const int rowb = fl ? 64 : 128;
    const int KS = mn ? rowb / 2 : rowb / esz;
    const int mnb = rowb / 2, boxb = rowb * KS;
    GemmTCDesc d{};
    d.M = M; d.N = N; d.K = K;
    // columns per CTA: the (padded) width up to 256, fewer while the stages do not fit the budget (bf16:
    // two stages and two CTAs per SM, so one tile's epilogue overlaps another's MMAs; the fp32 kinds three
    // stages and one CTA per SM, two TMEM buffers of up to 256 columns)
    const long long npad = mn ? (N + mnb - 1) / mnb * mnb : (N + 15) & ~15LL;
    const int budget = (fl ? 216 : 110) * 1024;
    const int min_stages = fl ? 3 : 2;
    d.a_bytes = 128 * rowb;
    const int ncap = fl ? 192 : 256;   // fp32 kinds: two TMEM buffers of <= 192 columns, 96 per epilogue thread
    int nc = (int)(npad <= ncap ? npad : ncap);
    for (;;) {
        d.b_bytes = mn ? ((nc + mnb - 1) / mnb) * boxb : nc * rowb;
        d.stage_bytes = NP * (d.a_bytes + d.b_bytes);
        if (min_stages * d.stage_bytes <= budget || nc <= 64) break;
        nc = mn ? nc - mnb : ((nc / 2 + 15) & ~15);
    }
    d.ncols_max = nc;
    d.tbuf = nc <= 128 ? 128 : 192;
    d.stages = budget / d.stage_bytes;
    if (d.stages > 6) d.stages = 6;
    if (d.stages < 2 || d.stages * d.stage_bytes < 128 * ((fl ? 192 : 128) + 1) * 4) return cudaErrorNotSupported;
    const long long kb_total = (K + KS - 1) / KS;
    d.kchunk = ((kb_total + nsplit - 1) / nsplit) * KS;
    d.kflush = g_kflush;
    d.D = D; d.ldd = ldd; d.split_stride = split_stride; d.status = status;
    const int dt = kind == KIND_TF32X3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap ma[3], mb[3];
    const int swz = fl ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    auto enc = [&](CUtensorMap* m, const void* p, long long rows, long long ld, unsigned boxrows) {
        if (mn) {   // [K, rows] row-major: inner dimension = rows
            const unsigned long long dims[2] = {(unsigned long long)rows, (unsigned long long)K};
            const unsigned long long str[1] = {(unsigned long long)(ld * esz)};
            const unsigned box[2] = {(unsigned)mnb, (unsigned)KS};
            return tmap_encode_ex(m, p, dt, 2, dims, str, box, swz);
        }
        const unsigned long long dims[2] = {(unsigned long long)K, (unsigned long long)rows};
        const unsigned long long str[1] = {(unsigned long long)(ld * esz)};
        const unsigned box[2] = {(unsigned)KS, boxrows};
        return tmap_encode_ex(m, p, dt, 2, dims, str, box, swz);
    };
    for (int p = 0; p < 3; p++) {
        if (p < NP) {
            if (!enc(&ma[p], A.p[p], M, A.ld, 128) || !enc(&mb[p], B.p[p], N, B.ld, (unsigned)d.ncols_max))
                return cudaErrorNotSupported;
        } else {
            ma[p] = ma[0];
            mb[p] = mb[0];
        }
    }
    const int smem = 1024 + d.stages * d.stage_bytes + (2 * d.stages + 5) * 8 + 16;
    const dim3 grid((unsigned)((npad + d.ncols_max - 1) / d.ncols_max), (unsigned)((M + 127) / 128), (unsigned)nsplit);
    if (grid.y > 65535u || grid.z > 65535u) return cudaErrorNotSupported;
    cudaError_t e = cudaErrorNotSupported;
#define KMB_GT(KI, EP, MNV)                                                                                 \
    do {                                                                                                    \
        e = cudaFuncSetAttribute(gemm_tc_kernel<KI, EP, MNV>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                 smem);                                                                     \
        if (e != cudaSuccess) return e;                                                                     \
        gemm_tc_kernel<KI, EP, MNV><<<grid, GT_THREADS, smem, st>>>(d, ma[0], ma[1], ma[2], mb[0],            \
                                                                              mb[1], mb[2]);                \
        e = cudaGetLastError();                                                                             \
    } while (0)
#define KMB_GT_EPI(KI, MNV)                      \
    do {                                         \
        if (epi == EPI_ADD) KMB_GT(KI, EPI_ADD, MNV); \
        else KMB_GT(KI, EPI_STORE, MNV);         \
    } while (0)
    switch (kind) {
        case KIND_BF16: if (mn) KMB_GT_EPI(KIND_BF16, true); else KMB_GT_EPI(KIND_BF16, false); break;
        case KIND_TF32X3: KMB_GT_EPI(KIND_TF32X3, false); break;
        case KIND_BF16X6: if (mn) KMB_GT_EPI(KIND_BF16X6, true); else KMB_GT_EPI(KIND_BF16X6, false); break;
        case KIND_BF16X9: if (mn) KMB_GT_EPI(KIND_BF16X9, true); else KMB_GT_EPI(KIND_BF16X9, false); break;
        default: return cudaErrorNotSupported;
    }
#undef KMB_GT_EPI
#undef KMB_GT
    return e;
}

// Pieces of an fp32 matrix [rows, cols] (row stride ldx) for `kind`, written with row stride ldo:
// TF32X3 into out[0..1] (fp32), BF16X6 / BF16X9 into out[0..2] (bf16).
cudaError_t gemm_split(int kind, const float* x, void* const* out, long long rows, long long cols, long long ldx,
                       long long ldo, cudaStream_t st) {
    if (rows * cols <= 0) return cudaSuccess;
    if (kind != KIND_TF32X3 && kind != KIND_BF16X6 && kind != KIND_BF16X9) return cudaErrorInvalidValue;
    // the four-column form may also split the row padding up to a multiple of 4 when both row strides
    // cover it: the GEMM's tensor maps stop at the true K, so padded pieces are never read
    const long long cols4 = (cols + 3) & ~3LL;
    bool vec = ldx % 4 == 0 && ldo % 4 == 0 && ldx >= cols4 && ldo >= cols4 && !((uintptr_t)x & 15);
    for (int p = 0; p < (kind == KIND_TF32X3 ? 2 : 3); p++) vec = vec && !((uintptr_t)out[p] & 15);
    if (vec) {
        const long long n = rows * (cols4 / 4);
        const unsigned g = (unsigned)((n + 255) / 256);
        if (kind == KIND_TF32X3)
            split_tf32<<<g, 256, 0, st>>>(x, (float*)out[0], (float*)out[1], rows, (int)(cols4 / 4), ldx, ldo);
        else
            split_bf16x3<<<g, 256, 0, st>>>(x, (__nv_bfloat16*)out[0], (__nv_bfloat16*)out[1],
                                            (__nv_bfloat16*)out[2], rows, (int)(cols4 / 4), ldx, ldo);
    } else {
        const long long n = rows * cols;
        split_any<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(kind, x, out[0], out[1], out[2], rows, cols, ldx, ldo);
    }
    return cudaGetLastError();
}

cudaError_t gemm_transpose_f32(const float* in, float* out, long long R, long long Cn, long long ldi, long long ldo,
                               cudaStream_t st) {
    dim3 grid((unsigned)((Cn + 31) / 32), (unsigned)((R + 31) / 32));
    transpose_2d<float><<<grid, dim3(32, 8), 0, st>>>(in, out, R, Cn, ldi, ldo);
    return cudaGetLastError();
}
cudaError_t gemm_transpose_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, long long R, long long Cn,
                                long long ldi, long long ldo, cudaStream_t st) {
    dim3 grid((unsigned)((Cn + 31) / 32), (unsigned)((R + 31) / 32));
    transpose_2d<__nv_bfloat16><<<grid, dim3(32, 8), 0, st>>>(in, out, R, Cn, ldi, ldo);
    return cudaGetLastError();
}

// out[r, c] (+)= sum over splits of part[s][r, c]
cudaError_t gemm_reduce_splits(const float* part, float* out, long long rows, long long cols, int nsplit,
                               long long split_stride, long long ldp, long long ldo, int accumulate, cudaStream_t st) {
    const long long n = rows * cols;
    gt_reduce_splits<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, out, n, nsplit, split_stride, accumulate, ldp,
                                                                   ldo, cols);
    return cudaGetLastError();
}

// MMA K steps of the leading product per TMEM flush of the fp32 kinds (1 .. 64); fewer = closer to
// fp32 FMA accuracy
int gemm_set_kflush(int k) {
    if (k < 1 || k > 64) return -1;
    g_kflush = k;
    return 0;
}

}  // namespace kmb
