// scannd_tma.cu -- persistent Scan-A forward for 1D grids on sm_100a (2D grids
// use the column-strip pipeline of scannd_strips.cu).  This file also holds the
// host-side TMA descriptor encoder shared by both kernels.
//
// Work decomposition
//   tile   = (item b, channel tile [d0, d0+DT)), DT*M = 256 recurrence lanes.
//   CTA    = 8 warps, one recurrence lane per thread (2 warps per SM
//            sub-partition, so each thread may hold up to 255 registers); the
//            grid is persistent (<= #SMs x resident CTAs) and walks tiles.
//   order  = the 2D grid is walked outer-by-inner (o, q), where the inner axis
//            is the shorter one (<= QT); it is causal for both predecessors:
//            (o, q-1) is the previous point and (o-1, q) was visited one outer
//            step earlier.  1D grids have no outer axis.
//   state  = per lane, the rotated state R h and the B*x product of the
//            previous outer row live in registers (ring[QT], fully unrolled),
//            so predecessor values never leave the SM and nothing but
//            B, C, x, delta, lambda (read once) and h, y (written once) touch
//            HBM: 12 B per state update + 4*(2+nd) B per (point, channel).
// Pipeline
//   stage  = G consecutive inner points of one tile: boxes of B and C
//            [G][DT][M], x [G][DT], delta [nd][G][DT] and lambda, fetched with
//            cp.async.bulk.tensor (plain, no multicast) into an NS-deep shared
//            memory ring guarded by mbarriers (full: TMA bytes landed; empty:
//            all 8 warps done).  Lane 0 of warp 0 issues the copies: before
//            each stage it tops the ring up to NS-1 stages ahead, blocking only
//            when the stage it is about to consume has not been issued yet.
//   y      = each lane stores C*h for the stage into a padded transposed
//            buffer; one consumer warp per stage (rotating) sums the M products
//            of each (point, channel) in ascending m and writes y, then frees
//            the stage.  All waits are mbarrier try_wait loops bounded by a
//            global-timer limit; on timeout the kernel writes an error code to
//            the status word and returns (the issuer first drains its copies).
#include <cuda.h>
#include "kmb_common.cuh"
#include "kmb_sync.cuh"

namespace kmb {
int persistent_sms(int sms);  // SMs a persistent grid may fill (capi.cu)

constexpr int TG = 8;      // points per stage
constexpr int TNS = 6;     // stages in the ring
constexpr int TNCW = 8;    // consumer warps
constexpr int TTHREADS = TNCW * 32;

struct FastDesc {
    int M, DT, D, nd;
    int Q, O;               // inner / outer extents (O = 1 for 1D)
    int k_in;               // axis index of the inner dimension
    int lam_inner_fast;     // lambda box (G,1,1) at (q0,o,b) vs (4,G,1) at (o&~3,q0,b)
    int has_lambda, fast_exp, clamp;
    float amin, deflam;
    long long qstride, ostride;  // point strides of the inner / outer dims
    long long P;
    int ntd;                // channel tiles per item (D / DT)
    long long ntiles;       // batch * ntd
    int sq_count;           // ceil(Q / G)
    unsigned tx_bytes;      // TMA bytes per stage
    const float* A;
    const float* theta;
    float* h;
    float* y;
    int* status;
};

// One state update of lane (d, m) at inner position q of outer row o.
// hasI/hasO: inner / outer predecessor present.  Returns h; writes the rotated
// state and B*x product for the successors through hat_out / bu_out.
template <bool ROPE>
__device__ __forceinline__ float scan_point(bool hasI, bool hasO, bool inner_is_axis0,
                                            float x, float dI, float dO, float lam, float Bv,
                                            float AI, float AO, int fast,
                                            float hatI, float buI, float hatO, float buO,
                                            float cth, float sth, bool odd,
                                            float& hat_out, float& bu_out) {
    const float dt = __fadd_rn(dI, dO);
    const float bu = __fmul_rn(Bv, x);
    float buacc = 0.0f, dacc = 0.0f, hacc = 0.0f, inv = 0.0f;
    if (hasI && hasO) {
        const float aI = kmb_exp(__fmul_rn(dI, AI), fast);
        const float aO = kmb_exp(__fmul_rn(dO, AO), fast);
        buacc = __fadd_rn(buI, buO);
        dacc = __fadd_rn(aI, aO);
        // axis-0 term first, as the reference accumulates in axis order
        hacc = inner_is_axis0 ? __fmaf_rn(aO, hatO, __fmul_rn(aI, hatI))
                              : __fmaf_rn(aI, hatI, __fmul_rn(aO, hatO));
        inv = 0.5f;
    } else if (hasI) {
        const float aI = kmb_exp(__fmul_rn(dI, AI), fast);
        buacc = buI;
        dacc = aI;
        hacc = __fmul_rn(aI, hatI);
        inv = 1.0f;
    } else if (hasO) {
        const float aO = kmb_exp(__fmul_rn(dO, AO), fast);
        buacc = buO;
        dacc = aO;
        hacc = __fmul_rn(aO, hatO);
        inv = 1.0f;
    }
    const float buavg = __fmul_rn(buacc, inv);  // exact: n is 1 or 2
    const float alavg = __fmul_rn(dacc, inv);
    const float beta = __fmul_rn(__fmul_rn(__fsub_rn(1.0f, lam), dt), alavg);
    const float gamma = __fmul_rn(lam, dt);
    const float hn = __fadd_rn(__fmaf_rn(bu, gamma, __fmul_rn(buavg, beta)), hacc);
    if (ROPE) {
        const float hp = __shfl_xor_sync(0xffffffffu, hn, 1);
        hat_out = odd ? __fmaf_rn(sth, hp, __fmul_rn(cth, hn)) : __fmaf_rn(cth, hn, -__fmul_rn(sth, hp));
    } else {
        hat_out = hn;
    }
    bu_out = bu;
    return hn;
}

template <int MT>
struct StageLayout {
    static constexpr int DT = 256 / MT;                 // channels per tile
    static constexpr int BBOX = TG * DT * MT * 4;       // bytes of one B / C box
    static constexpr int RS = TG * DT + 1;              // product buffer row stride (floats)
    static constexpr int offC = BBOX;
    static constexpr int offX = 2 * BBOX;
    static constexpr int offD = offX + ((TG * DT * 4 + 127) & ~127);
    static constexpr int offL = offD + ((2 * TG * DT * 4 + 127) & ~127);
    static constexpr int offP = offL + 128;
    static constexpr int bytes = (offP + MT * RS * 4 + 127) & ~127;
};

template <int NDIM, bool ROPE, int QT, int MT>
__global__ void __launch_bounds__(TTHREADS, 1)
scan_fwd_tma(const __grid_constant__ FastDesc f,
             const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mC,
             const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mD,
             const __grid_constant__ CUtensorMap mL) {
    using L = StageLayout<MT>;
    constexpr int DT = L::DT;
    constexpr int G = TG;
    constexpr int NP = G * DT;  // (point, channel) outputs per stage
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    unsigned char* stages = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)TNS * L::bytes);
    // bars[0..NS): full, [NS..2NS): empty, [2NS..3NS): products ready
    if (tid == 0) {
        for (int i = 0; i < TNS; i++) {
            mbar_init(smem_u32(&bars[i]), 1);
            mbar_init(smem_u32(&bars[TNS + i]), TNCW);
            mbar_init(smem_u32(&bars[2 * TNS + i]), TNCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const long long stages_per_tile = (long long)f.O * f.sq_count;

    // ------------------------------------------------------------- issuer
    // Stage t (a global sequence over this CTA's tiles) maps to
    // (tile_idx, o, sq); slot t % NS; its slot is free once stage t-NS is
    // released (empty barrier phase ((t/NS)-1) & 1).
    const long long total_stages = ((f.ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x) * stages_per_tile;
    long long next_issue = 0;
    const bool issuer = (warp == 0 && lane == 0);
    auto issue = [&](long long t) {
        const long long ti = t / stages_per_tile;
        const long long rem = t % stages_per_tile;
        const int o = (int)(rem / f.sq_count), sq = (int)(rem % f.sq_count);
        const long long tile = blockIdx.x + ti * gridDim.x;
        const int b = (int)(tile / f.ntd);
        const int d0 = (int)(tile % f.ntd) * DT;
        const int slot = (int)(t % TNS);
        unsigned char* st = stages + (size_t)slot * L::bytes;
        const uint32_t full = smem_u32(&bars[slot]);
        mbar_expect_tx(full, f.tx_bytes);
        const int q0 = sq * G;
        tma_load_5d(smem_u32(st), &mB, full, 0, d0, q0, o, b);
        tma_load_5d(smem_u32(st + L::offC), &mC, full, 0, d0, q0, o, b);
        tma_load_4d(smem_u32(st + L::offX), &mX, full, d0, q0, o, b);
        tma_load_5d(smem_u32(st + L::offD), &mD, full, d0, q0, o, 0, b);
        if (f.has_lambda) {
            if (f.lam_inner_fast) tma_load_3d(smem_u32(st + L::offL), &mL, full, q0, o, b);
            else tma_load_3d(smem_u32(st + L::offL), &mL, full, o & ~3, q0, b);
        }
    };
    // Lane 0 of warp 0, before consuming stage `cur`: keep up to NS stages in
    // flight; block only for the stage about to be consumed.  false = gave up.
    auto top_up = [&](long long cur) -> bool {
        while (next_issue < total_stages && next_issue < cur + TNS) {
            const long long t = next_issue;
            if (t >= TNS) {
                const uint32_t eb = smem_u32(&bars[TNS + (int)(t % TNS)]);
                const uint32_t ph = (uint32_t)(((t / TNS) - 1) & 1);
                if (t <= cur) {
                    if (!mbar_wait(eb, ph)) return false;
                } else if (!mbar_try(eb, ph)) {
                    break;
                }
            }
            issue(t);
            next_issue++;
        }
        return true;
    };
    auto drain = [&]() {  // wait (bounded) for copies still in flight
        if (!issuer) return;
        for (long long j = (next_issue > TNS ? next_issue - TNS : 0); j < next_issue; j++)
            mbar_wait(smem_u32(&bars[j % TNS]), (uint32_t)((j / TNS) & 1));
    };

    // ------------------------------------------------------------- lanes
    int dl, m;
    if (ROPE) {
        const int r = tid % (2 * MT);
        dl = 2 * (tid / (2 * MT)) + (r & 1);
        m = r >> 1;
    } else {
        dl = tid / MT;
        m = tid % MT;
    }
    const bool odd = (dl & 1) != 0;
    const int D = f.D;
    const int k_in = f.k_in;
    const bool inner_is_axis0 = (k_in == 0);
    const long long DM = (long long)D * MT;
    const long long hq = f.qstride * DM;  // h stride between consecutive inner points
    long long s = 0;

    for (long long tile = blockIdx.x; tile < f.ntiles; tile += gridDim.x) {
        const int b = (int)(tile / f.ntd);
        const int d0 = (int)(tile % f.ntd) * DT;
        const int d = d0 + dl;
        const float AI = kmb_clampA(f.A[((long long)k_in * D + d) * MT + m], f.clamp, f.amin);
        const float AO = (NDIM == 2) ? kmb_clampA(f.A[((long long)(1 - k_in) * D + d) * MT + m], f.clamp, f.amin) : 0.0f;
        float cth = 1.0f, sth = 0.0f;
        if (ROPE) {
            const float th = f.theta[d >> 1];
            kmb_cos_sin(th, &cth, &sth);
        }
        float* const hb = f.h + (long long)b * f.P * DM + (long long)d * MT + m;
        float* const yb = f.y + (long long)b * f.P * D + d0;
        float ring_h[QT], ring_b[QT];
        float hprev = 0.0f, buprev = 0.0f;

        // Wait for stage s, run `compute`, publish products, reduce y if this
        // warp owns the stage, release it.  false = gave up (status written).
        auto run_stage = [&](int o, int sq, auto compute) -> bool {
            const int slot = (int)(s % TNS);
            const uint32_t ph = (uint32_t)((s / TNS) & 1);
            if (issuer && !top_up(s)) {
                set_status(f.status, KMB_ERR_TIMEOUT_EMPTY);
                drain();
                return false;
            }
            __syncwarp();
            if (!mbar_wait(smem_u32(&bars[slot]), ph)) {
                set_status(f.status, KMB_ERR_TIMEOUT_FULL);
                drain();
                return false;
            }
            const unsigned char* st = stages + (size_t)slot * L::bytes;
            float* prod = (float*)(stages + (size_t)slot * L::bytes + L::offP);
            compute(st, prod);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars[2 * TNS + slot]));
            if (warp == (int)(s % TNCW)) {
                if (!mbar_wait(smem_u32(&bars[2 * TNS + slot]), ph)) {
                    set_status(f.status, KMB_ERR_TIMEOUT_Y);
                    drain();
                    return false;
                }
                float* yrow = yb + ((long long)o * f.ostride + (long long)sq * G * f.qstride) * D;
#pragma unroll 1
                for (int j = lane; j < NP; j += 32) {
                    const int g = j / DT, c = j % DT;
                    if (sq * G + g < f.Q) {
                        float acc = 0.0f;
#pragma unroll 8
                        for (int mm = 0; mm < MT; mm++) acc = __fadd_rn(acc, prod[mm * L::RS + j]);
                        yrow[(long long)g * f.qstride * D + c] = acc;
                    }
                }
                __syncwarp();
            }
            if (lane == 0) mbar_arrive(smem_u32(&bars[TNS + slot]));
            s++;
            return true;
        };

        // One state update at stage-local point g.  hp: h address of the point.
        auto point = [&](const unsigned char* st, float* prod, int g, int o, float* hp, bool hasI,
                         bool hasO, float hatI, float buI, float hatO, float buO, float& hat_out,
                         float& bu_out) {
            const float* Bs = (const float*)st;
            const float* Xs = (const float*)(st + L::offX);
            const float* Ds = (const float*)(st + L::offD);
            const float* Ls = (const float*)(st + L::offL);
            const float* Cs = (const float*)(st + L::offC);
            const int row = g * DT + dl;
            const float x = Xs[row];
            const float dI = Ds[k_in * NP + row];
            const float dO = (NDIM == 2) ? Ds[(1 - k_in) * NP + row] : 0.0f;
            const float lam = f.has_lambda ? (f.lam_inner_fast ? Ls[g] : Ls[g * 4 + (o & 3)]) : f.deflam;
            const float Bv = Bs[row * MT + m];
            const float Cv = Cs[row * MT + m];
            const float hn = scan_point<ROPE>(hasI, hasO, inner_is_axis0, x, dI, dO, lam, Bv, AI, AO,
                                              f.fast_exp, hatI, buI, hatO, buO, cth, sth, odd, hat_out, bu_out);
            __stcs(hp, hn);
            prod[m * L::RS + row] = __fmul_rn(Cv, hn);
        };

        if constexpr (NDIM == 1) {
            float* hp = hb;
#pragma unroll 1
            for (int sq = 0; sq < f.sq_count; sq++) {
                const bool okst = run_stage(0, sq, [&](const unsigned char* st, float* prod) {
#pragma unroll
                    for (int g = 0; g < TG; g++) {
                        const int q = sq * TG + g;
                        if (q < f.Q) {
                            float ho, bo;
                            point(st, prod, g, 0, hp, q > 0, false, hprev, buprev, 0.0f, 0.0f, ho, bo);
                            hprev = ho;
                            buprev = bo;
                            hp += hq;
                        }
                    }
                });
                if (!okst) return;
            }
        } else {
#pragma unroll 1
            for (int o = 0; o < f.O; o++) {
                const bool hasO = o > 0;
                float* hp = hb + (long long)o * f.ostride * DM;
#pragma unroll
                for (int sq = 0; sq < QT / TG; sq++) {
                    if (sq < f.sq_count) {
                        const bool okst = run_stage(o, sq, [&](const unsigned char* st, float* prod) {
#pragma unroll
                            for (int g = 0; g < TG; g++) {
                                const int q = sq * TG + g;
                                if (q < f.Q) {
                                    float ho, bo;
                                    point(st, prod, g, o, hp, q > 0, hasO,
                                          ring_h[q > 0 ? q - 1 : 0], ring_b[q > 0 ? q - 1 : 0],
                                          ring_h[q], ring_b[q], ho, bo);
                                    ring_h[q] = ho;
                                    ring_b[q] = bo;
                                    hp += hq;
                                }
                            }
                        });
                        if (!okst) return;
                    }
                }
            }
        }
        (void)hprev;
        (void)buprev;
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
    static PFN_encodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_encodeTiled)p;
    }
    return fn;
}

// Tiled tensor map of any element type and swizzle (no interleave; OOB elements read as zero)
bool tmap_encode_ex(CUtensorMap* m, const void* base, int dtype, int rank, const unsigned long long* dims,
                    const unsigned long long* strides_bytes, const unsigned* box, int swizzle) {
    PFN_encodeTiled fn = get_encode();
    if (!fn) return false;
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; i++) {
        gd[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i < rank - 1) gs[i] = strides_bytes[i];
    }
    CUresult r = fn(m, (CUtensorMapDataType)dtype, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool tmap_encode(CUtensorMap* m, const void* base, int rank, const unsigned long long* dims,
                 const unsigned long long* strides_bytes, const unsigned* box) {
    return tmap_encode_ex(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, dims, strides_bytes, box,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
}


template <int NDIM, bool ROPE, int QT, int MT>
static cudaError_t launch_inst(const FastDesc& f, const CUtensorMap* maps, cudaStream_t st) {
    auto k = scan_fwd_tma<NDIM, ROPE, QT, MT>;
    const int smem = TNS * StageLayout<MT>::bytes + 3 * TNS * 8;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev, sms, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sms = persistent_sms(sms);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, TTHREADS, smem);
    if (per < 1) return cudaErrorNotSupported;
    long long grid = (long long)sms * per;
    if (grid > f.ntiles) grid = f.ntiles;
    k<<<(unsigned)grid, TTHREADS, smem, st>>>(f, maps[0], maps[1], maps[2], maps[3], maps[4]);
    return cudaGetLastError();
}

template <int MT>
static cudaError_t dispatch_nd(const ScanDesc& s, const FastDesc& f, const CUtensorMap* maps, int QT,
                               cudaStream_t st) {
    (void)QT;
    return s.rope ? launch_inst<1, true, 1, MT>(f, maps, st) : launch_inst<1, false, 1, MT>(f, maps, st);
}

// Returns cudaErrorNotSupported when the shape is outside the fast path's
// envelope (the caller then uses the generic kernels).
cudaError_t launch_scan_fwd_tma(const ScanDesc& s, int* status, cudaStream_t st) {
    if (s.nd != 1) return cudaErrorNotSupported;
    const int M = s.M, D = s.D;
    if (M != 16 && M != 32 && M != 64) return cudaErrorNotSupported;
    const int DT = 256 / M;
    if (DT < 4 || D % DT != 0) return cudaErrorNotSupported;
    if (s.rope && (DT & 1)) return cudaErrorNotSupported;
    if (s.batch > 0x7fffffff || s.P > 0x7fffffffLL) return cudaErrorNotSupported;
    FastDesc f{};
    f.M = M; f.DT = DT; f.D = D; f.nd = (int)s.nd;
    const long long H = s.dims[0];
    const long long W = s.nd == 2 ? s.dims[1] : 1;
    int QT;
    if (s.nd == 1) {
        f.Q = (int)H; f.O = 1; f.k_in = 0; f.qstride = 1; f.ostride = H; f.lam_inner_fast = 1;
        QT = 1;
    } else {
        if (W <= 64) {        // rows: inner = axis 1
            f.Q = (int)W; f.O = (int)H; f.k_in = 1; f.qstride = 1; f.ostride = W; f.lam_inner_fast = 1;
        } else if (H <= 64) { // columns: inner = axis 0
            f.Q = (int)H; f.O = (int)W; f.k_in = 0; f.qstride = W; f.ostride = 1; f.lam_inner_fast = 0;
        } else {
            return cudaErrorNotSupported;
        }
        QT = f.Q <= 32 ? 32 : 64;
    }
    if (s.has_lambda && (W % 4) != 0 && s.nd == 2) return cudaErrorNotSupported;
    if (s.has_lambda && s.nd == 1 && (s.P % 4) != 0) return cudaErrorNotSupported;
    f.has_lambda = s.has_lambda; f.fast_exp = s.fast_exp; f.clamp = s.clamp;
    f.amin = s.a_log_min; f.deflam = s.default_lambda;
    f.P = s.P;
    f.ntd = D / DT;
    f.ntiles = s.batch * f.ntd;
    f.sq_count = (f.Q + TG - 1) / TG;
    const int bbox = TG * DT * M * 4;
    f.tx_bytes = (unsigned)(2 * bbox + TG * DT * 4 + s.nd * TG * DT * 4 +
                            (s.has_lambda ? (f.lam_inner_fast ? TG * 4 : 4 * TG * 4) : 0));
    f.A = s.A; f.theta = s.theta; f.h = s.h; f.y = s.y; f.status = status;

    // tensor maps: element strides in bytes of the (inner q, outer o) view
    const unsigned long long P = s.P, Bn = s.batch, DM = (unsigned long long)D * M;
    const unsigned long long qs = f.qstride, os = f.ostride;
    CUtensorMap maps[5];
    memset(maps, 0, sizeof(maps));
    {
        const unsigned long long dims[5] = {(unsigned long long)M, (unsigned long long)D,
                                            (unsigned long long)f.Q, (unsigned long long)f.O, Bn};
        const unsigned long long str[4] = {(unsigned long long)M * 4, qs * DM * 4, os * DM * 4, P * DM * 4};
        const unsigned box[5] = {(unsigned)M, (unsigned)DT, (unsigned)TG, 1, 1};
        if (!tmap_encode(&maps[0], s.B, 5, dims, str, box)) return cudaErrorNotSupported;
        if (!tmap_encode(&maps[1], s.C, 5, dims, str, box)) return cudaErrorNotSupported;
    }
    {
        const unsigned long long dims[4] = {(unsigned long long)D, (unsigned long long)f.Q,
                                            (unsigned long long)f.O, Bn};
        const unsigned long long str[3] = {qs * D * 4, os * D * 4, P * D * 4};
        const unsigned box[4] = {(unsigned)DT, (unsigned)TG, 1, 1};
        if (!tmap_encode(&maps[2], s.x, 4, dims, str, box)) return cudaErrorNotSupported;
    }
    {
        const unsigned long long dims[5] = {(unsigned long long)D, (unsigned long long)f.Q,
                                            (unsigned long long)f.O, (unsigned long long)s.nd, Bn};
        const unsigned long long str[4] = {qs * D * 4, os * D * 4, P * D * 4,
                                           (unsigned long long)s.nd * P * D * 4};
        const unsigned box[5] = {(unsigned)DT, (unsigned)TG, 1, (unsigned)s.nd, 1};
        if (!tmap_encode(&maps[3], s.delta, 5, dims, str, box)) return cudaErrorNotSupported;
    }
    if (s.has_lambda) {
        const unsigned long long dims[3] = {(unsigned long long)W, (unsigned long long)(s.nd == 2 ? H : 1), Bn};
        unsigned long long d0 = s.nd == 2 ? W : H;
        const unsigned long long dims1[3] = {d0, (unsigned long long)(s.nd == 2 ? H : 1), Bn};
        (void)dims;
        const unsigned long long str[2] = {d0 * 4, P * 4};
        const unsigned box[3] = {f.lam_inner_fast ? (unsigned)TG : 4u, f.lam_inner_fast ? 1u : (unsigned)TG, 1};
        if (!tmap_encode(&maps[4], s.lambda, 3, dims1, str, box)) return cudaErrorNotSupported;
    } else {
        maps[4] = maps[2];
    }
    if (M == 16) return dispatch_nd<16>(s, f, maps, QT, st);
    if (M == 32) return dispatch_nd<32>(s, f, maps, QT, st);
    return dispatch_nd<64>(s, f, maps, QT, st);
}

}  // namespace kmb
