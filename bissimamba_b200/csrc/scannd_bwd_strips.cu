// scannd_bwd_strips.cu -- exact Scan-A adjoint for 2D grids on sm_100a: a
// reverse systolic column-strip pipeline (the backward of the headline
// geometry, 2D 64x64, D=512, M=64, and of BASELINE config 1).
//
// The forward of src/scan_nd.c:103-201 at point p with predecessors p - e_k:
//   h(p) = sum_k a_k R h(p-e_k) + (1-lam) dt (sum_k a_k / n) (sum_k Bu(p-e_k) / n) + lam dt Bu(p)
// with a_k = exp(delta_k A_k), dt = sum_k delta_k, Bu = B x, n = #predecessors.
// Its adjoint is a recurrence running the other way: the state gradient of p
// depends only on p's successors s_k = p + e_k,
//   g_h(p)  = C dy + R^T sum_k P_k(s_k),      P_k(s) = a_k(s) g_h(s)
//   g_Bu(p) = lam dt g_h(p) + sum_k Q(s_k),   Q(s) = (1-lam(s)) dt(s) mean_a(s) g_h(s) / n(s)
// so every point passes (P_k, Q) to its predecessor along axis k.
//
// Work split (mirrors the forward strips kernel): a CTA owns a tile (item b,
// CH channels, 32 states; M = 64 runs as two tiles of 32 states), the inner
// axis (<= 64 columns) is cut into strips of 8 columns with one warp per strip,
// and each lane carries two channels (the RoPE pair, or two independent
// channels) of one state.  Rows are walked bottom to top and, within a row,
// columns right to left.  The (P_in, Q) of a strip's first column goes to the
// warp on its left through mbarrier-guarded shared-memory slots; the
// (P_out, Q) of every column stays in registers for the row above.  Strips run
// one row apart, so no adjoint is ever written to or read back from memory
// (the level-parallel kernel's G scratch is gone).
//
// Per lane, h and B of three rows are in registers: the current row (own
// values), the row above (the up-predecessors' values, loaded one row ahead)
// and the row above that (in flight).  The left predecessor is the next column
// of the same registers (its strip neighbour's last column at the strip edge,
// loaded once per row).  The per-(point, channel) inputs x, delta, dy and
// lambda go through a three-row shared-memory ring filled by cp.async.
//
// Sums over the states (ddelta, dx; dlambda also over the channels) are
// written per column to a padded shared-memory table and added in a fixed
// order at the end of each row; with M = 64 the two state halves leave
// partials that a second kernel adds in a fixed order.  dA and dtheta leave
// per-(item, strip) partials.  Everything is deterministic; dB, dC, ddelta, dx
// and dlambda are accumulated (+=, one addition per element) or, with
// overwrite, assigned.
//
// Traffic: reads h, B, C (12 B per state update) and, when accumulating,
// dB, dC (8 B), writes dB, dC (8 B): 28 B (20 B with overwrite) per update,
// plus x, delta, dy, lambda and ddelta, dx per (point, channel).
#include "kmb_common.cuh"
#include "kmb_sync.cuh"
#include <stdlib.h>
#include <type_traits>

namespace kmb {
int persistent_sms(int sms);  // SMs a persistent grid may fill (capi.cu)

// packed fp32 pairs (per component exactly __fadd_rn / __fmul_rn / __fmaf_rn)
__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

constexpr int BS_K = 4;    // handoff slots per strip boundary

struct BwdStripDesc {
    int D, Q, O, S;         // channels, columns, rows, strips
    int ntd;                // channel tiles per item
    long long ntiles;       // batch * ntd * G
    int has_lambda, clamp;
    float amin, deflam;
    long long P;
    const float *x, *A, *B, *C, *delta, *theta, *lambda, *h, *dy;
    float *dB, *dC, *ddelta, *dx;
    float* part;            // G > 1: [b][p][d][G][3] partial sums (ddelta inner, ddelta outer, dx)
    float *pA, *pth, *plam; // [b*S + w][2][D][M], [(b*G + g)*S + w][D/2], [b][ntd*G][P]
    int* status;
};

template <int M, int WC>
struct BsGeom {
    static constexpr int MS = M == 16 ? 16 : 32;      // states of one tile
    static constexpr int G = M / MS;                  // state halves (2 when M = 64)
    static constexpr int SETS = 32 / MS;              // channel sets per warp (2 when M = 16)
    static constexpr int CH = 2 * SETS;               // channels per tile
    // small per-row inputs in the cp.async ring: x [WC+1][CH], dI, dO, dy [WC][CH], lam [WC]
    static constexpr int XO = 0, DIO = (WC + 1) * CH, DOO = DIO + WC * CH, DYO = DOO + WC * CH,
                         LO = DYO + WC * CH, SMALL = (LO + WC + 3) / 4 * 4;
    static constexpr int NSL = (SMALL + 31) / 32;    // small loads per lane per row
    // per-row reduction table: rows (j, k) k = ddelta inner, ddelta outer, dx (two floats per lane)
    // and (j, 3) = dlambda (one float per lane); padded so 8 readers of 8 rows hit distinct banks
    static constexpr int RS = 68;
    static constexpr int ROWS = WC * 4;
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int M, bool ROPE, bool OVW, int WC>
__global__ void __launch_bounds__(WC == 8 ? 256 : 512, 1) scan_bwd_strips(const __grid_constant__ BwdStripDesc f) {
    using Gm = BsGeom<M, WC>;
    constexpr int CH = Gm::CH, SM_ = Gm::SMALL, MS = Gm::MS, G = Gm::G, RS = Gm::RS;
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int S = f.S, D = f.D, Q = f.Q, O = f.O, ntd = f.ntd;
    const long long P = f.P;
    // smem: small ring [S][3][SMALL] | reduction table [S][ROWS][RS] | handoff [S][K][2][32][2] | barriers
    float* small = (float*)smem;
    float* redt = small + S * 3 * SM_;
    float* hand = redt + S * Gm::ROWS * RS;
    uint64_t* bars = (uint64_t*)(hand + S * BS_K * 2 * 64);
    uint64_t* b_full = bars;                // [S][K]  boundary w: written by strip w, read by strip w-1
    uint64_t* b_empty = bars + S * BS_K;    // [S][K]
    if (tid == 0) {
        for (int i = 0; i < S * BS_K; i++) {
            mbar_init(smem_u32(&b_full[i]), 1);
            mbar_init(smem_u32(&b_empty[i]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (w >= S) return;

    const int set = lane / MS, ml = lane % MS;     // channel set, state within the tile
    const int cl0 = 2 * set;                       // first local channel of this lane
    const int q0 = w * WC;
    const int ncol = min(WC, Q - q0);
    float* my_small = small + w * 3 * SM_;
    float* my_red = redt + w * Gm::ROWS * RS;
    const int DM = D * M;                          // item-local offsets are 32-bit (P * D * M < 2^31)
    const int ngl = ntd * G;

    // per-lane small-load plan (relative to the item base and the row): array, column, channel
    int sl_off[Gm::NSL];
    int sl_kind[Gm::NSL];  // 0 x, 1 delta inner, 2 delta outer, 3 dy, 4 lambda, -1 none
#pragma unroll
    for (int t = 0; t < Gm::NSL; t++) {
        const int i = lane + 32 * t;
        sl_kind[t] = -1;
        sl_off[t] = 0;
        if (i < Gm::DIO) {
            const int j = i / CH - 1, c = i % CH;   // column -1 .. WC-1
            if (q0 + j >= 0 && j < ncol) { sl_kind[t] = 0; sl_off[t] = (q0 + j) * D + c; }
        } else if (i < Gm::LO) {
            const int r = i - Gm::DIO, a = r / (WC * CH), j = (r % (WC * CH)) / CH, c = r % CH;
            if (j < ncol) { sl_kind[t] = 1 + a; sl_off[t] = (q0 + j) * D + c; }
        } else if (i < SM_) {
            const int j = i - Gm::LO;
            if (j < ncol && f.has_lambda) { sl_kind[t] = 4; sl_off[t] = q0 + j; }
        }
    }

    int row = 0;  // global row counter of this warp (handoff slot / phase)
    for (long long tile = blockIdx.x; tile < f.ntiles; tile += gridDim.x) {
        const int half = (int)(tile % G);
        const long long bt = tile / G;
        const int b = (int)(bt / ntd);
        const int dt0 = (int)(bt - (long long)b * ntd);
        const int d0 = dt0 * CH;
        const int mg = half * 32 + ml;           // state index
        const int dl0 = d0 + cl0;                // first channel of this lane
        const long long ib = (long long)b * P * DM;
        const int lofs = dl0 * M + mg + q0 * DM;  // this lane's offset in a row at column q0
        const float* hb = f.h + ib + lofs;
        const float* Bb = f.B + ib + lofs;
        const float* Cb = f.C + ib + lofs;
        float* dBb = f.dB + ib + lofs;
        float* dCb = f.dC + ib + lofs;
        const float* xb = f.x + (long long)b * P * D + d0;
        const float* dlb = f.delta + (long long)b * 2 * P * D + d0;
        const float* dyb = f.dy + (long long)b * P * D + d0;
        const float* lb = f.has_lambda ? f.lambda + (long long)b * P : nullptr;
        const int rowDM = Q * DM;   // one row of h / B / C
        float AI[2], AO[2], AIL[2], AOL[2];
        bool clI[2], clO[2];
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int d = dl0 + c;
            const float ai = f.A[((long long)1 * D + d) * M + mg], ao = f.A[((long long)0 * D + d) * M + mg];
            clI[c] = f.clamp && ai > f.amin;
            clO[c] = f.clamp && ao > f.amin;
            AI[c] = clI[c] ? f.amin : ai;
            AO[c] = clO[c] ? f.amin : ao;
            // alpha = 2^(delta * A log2 e): one multiply and one ex2 per alpha
            AIL[c] = __fmul_rn(AI[c], kKmbLog2e);
            AOL[c] = __fmul_rn(AO[c], kKmbLog2e);
        }
        float cth = 1.0f, sth = 0.0f;
        if (ROPE) {
            const float th = f.theta[dl0 >> 1];
            kmb_cos_sin(th, &cth, &sth);
        }
        // state ring: own row (o), predecessor row (o-1), row in flight (o-2)
        float hO[WC][2], bO[WC][2], hP[WC][2], bP[WC][2], hN[WC][2], bN[WC][2], cO[WC][2], cN[WC][2];
        auto load_hb = [&](int o, float (&hh)[WC][2], float (&bb)[WC][2]) {
            const int ro = o * rowDM;
#pragma unroll
            for (int j = 0; j < WC; j++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const bool ok = j < ncol && o >= 0;
                    hh[j][c] = ok ? __ldg(hb + (ro + j * DM + c * M)) : 0.0f;
                    bb[j][c] = ok ? __ldg(Bb + (ro + j * DM + c * M)) : 0.0f;
                }
        };
        auto load_c = [&](int o, float (&cc)[WC][2]) {
            const int ro = o * rowDM;
#pragma unroll
            for (int j = 0; j < WC; j++)
#pragma unroll
                for (int c = 0; c < 2; c++)
                    cc[j][c] = (j < ncol && o >= 0) ? __ldg(Cb + (ro + j * DM + c * M)) : 0.0f;
        };
        auto load_small = [&](int o) {
            if (o < 0) return;
            float* dst = my_small + (o % 3) * SM_;
#pragma unroll
            for (int t = 0; t < Gm::NSL; t++) {
                const int k = sl_kind[t];
                if (k < 0) continue;
                const float* src = k == 0 ? xb : k == 1 ? dlb + P * D : k == 2 ? dlb : k == 3 ? dyb : lb;
                const int rs = k == 4 ? Q : Q * D;
                cp_async4(smem_u32(dst + lane + 32 * t), src + (o * rs + sl_off[t]));
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        // prologue: rows O-1 (own) and O-2 (predecessors)
        load_hb(O - 1, hO, bO);
        load_hb(O - 2, hP, bP);
        load_c(O - 1, cO);
        load_small(O - 1);
        load_small(O - 2);
        float dP[WC][2], dQ[WC][2];
#pragma unroll
        for (int j = 0; j < WC; j++) dP[j][0] = dP[j][1] = dQ[j][0] = dQ[j][1] = 0.0f;
        float gAI[2] = {0.f, 0.f}, gAO[2] = {0.f, 0.f}, gth = 0.0f;

        // one row; HASU: the row above exists (o > 0)
        auto do_row = [&](auto hasU_c, int o) -> bool {
            constexpr bool HASU = decltype(hasU_c)::value;
            cp_async_wait_all();
            __syncwarp();
            // issue the row after next: h, B of o-2; C of o-1; small inputs of o-2
            load_hb(o - 2, hN, bN);
            load_c(o - 1, cN);
            load_small(o - 2);
            const int ro = o * rowDM;
            float hL[2] = {0.f, 0.f}, bL[2] = {0.f, 0.f};
            if (q0 > 0) {
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    hL[c] = __ldg(hb + (ro - DM + c * M));
                    bL[c] = __ldg(Bb + (ro - DM + c * M));
                }
            }
            const float* sO = my_small + (o % 3) * SM_;
            const float* sP = my_small + ((o + 2) % 3) * SM_;   // row o-1
            const int hs = row & (BS_K - 1);
            const uint32_t hph = (uint32_t)((row / BS_K) & 1);
            // right successor of the last column: strip w+1's first column
            float rP[2] = {0.f, 0.f}, rQ[2] = {0.f, 0.f};
            if (w + 1 < S) {
                if (!mbar_wait(smem_u32(&b_full[(w + 1) * BS_K + hs]), hph)) {
                    set_status(f.status, KMB_ERR_TIMEOUT_Y);
                    return false;
                }
                const float2* src = (const float2*)(hand + ((size_t)((w + 1) * BS_K + hs) * 2) * 64);
                const float2 pv = src[lane], qv = src[32 + lane];
                rP[0] = pv.x; rP[1] = pv.y;
                rQ[0] = qv.x; rQ[1] = qv.y;
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&b_empty[(w + 1) * BS_K + hs]));
            }
            // x of column j as (channel c0, c0 + 1); the left predecessor's x is the next column's own
            float2 xr = *(const float2*)(sO + Gm::XO + (WC) * CH + cl0);
#pragma unroll
            for (int j = WC - 1; j >= 0; j--) {
                if (j >= ncol) {
                    if (j > 0) xr = *(const float2*)(sO + Gm::XO + j * CH + cl0);
                    continue;
                }
                const bool hasL = j > 0 || q0 > 0;
                const float lam = f.has_lambda ? sO[Gm::LO + j] : f.deflam;
                const float inv = (HASU && hasL) ? 0.5f : 1.0f;
                const float2 xo = xr;                                                   // own x
                const float2 xl = *(const float2*)(sO + Gm::XO + j * CH + cl0);         // left x
                xr = xl;
                const float2 xu = *(const float2*)(sP + Gm::XO + (j + 1) * CH + cl0);   // up x
                const float2 dI2 = *(const float2*)(sO + Gm::DIO + j * CH + cl0);
                const float2 dO2 = *(const float2*)(sO + Gm::DOO + j * CH + cl0);
                const float2 dy2 = *(const float2*)(sO + Gm::DYO + j * CH + cl0);
                // Both channels of the lane as packed fp32 pairs (.x = channel dl0, .y = dl0 + 1): the
                // same IEEE operations per channel as a scalar loop over the two, half the instructions.
                const float2 ah2 = f2add(make_float2(rP[0], rP[1]), make_float2(dP[j][0], dP[j][1]));
                const float2 ab2 = f2add(make_float2(rQ[0], rQ[1]), make_float2(dQ[j][0], dQ[j][1]));
                const float2 h2 = make_float2(hO[j][0], hO[j][1]);
                const float2 lh2 = j > 0 ? make_float2(hO[j > 0 ? j - 1 : 0][0], hO[j > 0 ? j - 1 : 0][1])
                                         : make_float2(hL[0], hL[1]);
                // R v for the pair v: (cth v0 - sth v1, sth v0 + cth v1); R^T a: (cth a0 + sth a1, cth a1 - sth a0)
                auto rot = [&](float2 v) {
                    const float2 m = f2mul(make_float2(sth, cth), make_float2(v.y, v.y));
                    return f2fma(make_float2(cth, sth), make_float2(v.x, v.x), make_float2(-m.x, m.y));
                };
                float2 gh2;
                if (ROPE) {
                    const float2 m = f2mul(make_float2(sth, sth), make_float2(ah2.y, ah2.x));
                    gh2 = f2fma(make_float2(cth, cth), ah2, make_float2(m.x, -m.y));
                    const float2 hat = rot(h2);
                    gth = __fmaf_rn(ah2.y, hat.x, __fmaf_rn(-ah2.x, hat.y, gth));
                } else {
                    gh2 = ah2;
                }
                const float oml = __fsub_rn(1.0f, lam);
                const float2 oml2 = make_float2(oml, oml), lam2 = make_float2(lam, lam);
                const float2 B2 = make_float2(bO[j][0], bO[j][1]);
                const float2 g2 = f2fma(make_float2(cO[j][0], cO[j][1]), dy2, gh2);
                const float2 dt2 = f2add(dO2, dI2);
                const float2 bu2 = f2mul(B2, xo);
                const float2 gam2 = f2mul(lam2, dt2);
                float2 gdt2 = f2mul(f2mul(lam2, bu2), g2);
                float2 gl2 = f2mul(f2mul(dt2, bu2), g2);
                const float2 z2 = make_float2(0.0f, 0.0f);
                float2 PI2 = z2, PO2 = z2, Qv2 = z2, eI2 = z2, eO2 = z2;
                if (HASU || hasL) {
                    float2 aI2 = z2, aO2 = z2, sbu2 = z2, hatL2 = z2, hatU2 = z2;
                    if (hasL) {
                        const float2 za = f2mul(dI2, make_float2(AIL[0], AIL[1]));
                        aI2 = make_float2(kmb_ex2(za.x), kmb_ex2(za.y));
                        const float2 bl2 = j > 0 ? make_float2(bO[j > 0 ? j - 1 : 0][0], bO[j > 0 ? j - 1 : 0][1])
                                                 : make_float2(bL[0], bL[1]);
                        sbu2 = f2mul(bl2, xl);
                        hatL2 = ROPE ? rot(lh2) : lh2;
                    }
                    if (HASU) {
                        const float2 za = f2mul(dO2, make_float2(AOL[0], AOL[1]));
                        aO2 = make_float2(kmb_ex2(za.x), kmb_ex2(za.y));
                        sbu2 = f2fma(make_float2(bP[j][0], bP[j][1]), xu, sbu2);
                        const float2 u2 = make_float2(hP[j][0], hP[j][1]);
                        hatU2 = ROPE ? rot(u2) : u2;
                    }
                    const float2 inv2 = make_float2(inv, inv);
                    const float2 ma2 = f2mul(f2add(aI2, aO2), inv2);   // mean alpha
                    const float2 mb2 = f2mul(sbu2, inv2);                 // mean predecessor Bu
                    const float2 omdt2 = f2mul(oml2, dt2);
                    PI2 = f2mul(aI2, g2);
                    PO2 = f2mul(aO2, g2);
                    Qv2 = f2mul(f2mul(f2mul(omdt2, ma2), inv2), g2);
                    const float2 mab2 = f2mul(ma2, mb2);
                    gdt2 = f2fma(f2mul(oml2, mab2), g2, gdt2);
                    const float2 dm = f2mul(dt2, mab2);
                    gl2 = f2fma(make_float2(-dm.x, -dm.y), g2, gl2);
                    const float2 ka2 = f2mul(f2mul(omdt2, inv2), mb2);   // d h / d a_k beyond the state term
                    if (hasL) {
                        const float2 dz = f2mul(PI2, f2add(hatL2, ka2));   // (d a / d z) g (...) with d a / d z = a
                        eI2 = f2mul(dz, make_float2(AI[0], AI[1]));
                        const float2 t = f2fma(dz, dI2, make_float2(gAI[0], gAI[1]));
                        gAI[0] = clI[0] ? gAI[0] : t.x;
                        gAI[1] = clI[1] ? gAI[1] : t.y;
                    }
                    if (HASU) {
                        const float2 dz = f2mul(PO2, f2add(hatU2, ka2));
                        eO2 = f2mul(dz, make_float2(AO[0], AO[1]));
                        const float2 t = f2fma(dz, dO2, make_float2(gAO[0], gAO[1]));
                        gAO[0] = clO[0] ? gAO[0] : t.x;
                        gAO[1] = clO[1] ? gAO[1] : t.y;
                    }
                }
                const float2 gbu2 = f2fma(gam2, g2, ab2);
                const float2 vC = f2mul(dy2, h2), vB = f2mul(gbu2, xo);
                {
                    const int eo = ro + j * DM;
                    if (OVW) {
                        __stcs(dCb + eo, vC.x);
                        __stcs(dBb + eo, vB.x);
                        __stcs(dCb + eo + M, vC.y);
                        __stcs(dBb + eo + M, vB.y);
                    } else {
                        atomicAdd(dCb + eo, vC.x);
                        atomicAdd(dBb + eo, vB.x);
                        atomicAdd(dCb + eo + M, vC.y);
                        atomicAdd(dBb + eo + M, vB.y);
                    }
                }
                const float2 reI = f2add(eI2, gdt2), reO = f2add(eO2, gdt2), rgx = f2mul(gbu2, B2);
                const float glam_l = __fadd_rn(__fadd_rn(0.0f, gl2.x), gl2.y);
                // pass to the predecessors: (P_in, Q) left, (P_out, Q) up
                dP[j][0] = PO2.x; dP[j][1] = PO2.y;
                dQ[j][0] = Qv2.x; dQ[j][1] = Qv2.y;
                rP[0] = PI2.x; rP[1] = PI2.y;
                rQ[0] = Qv2.x; rQ[1] = Qv2.y;
                const float red_eI[2] = {reI.x, reI.y}, red_eO[2] = {reO.x, reO.y}, red_gx[2] = {rgx.x, rgx.y};
                float* rr = my_red + (j * 4) * RS;
                *(float2*)(rr + 0 * RS + 2 * lane) = make_float2(red_eI[0], red_eI[1]);
                *(float2*)(rr + 1 * RS + 2 * lane) = make_float2(red_eO[0], red_eO[1]);
                *(float2*)(rr + 2 * RS + 2 * lane) = make_float2(red_gx[0], red_gx[1]);
                rr[3 * RS + lane] = glam_l;
            }
            // left edge: hand (P_in, Q) of column q0 to strip w-1
            if (w > 0) {
                if (row >= BS_K && !mbar_wait(smem_u32(&b_empty[w * BS_K + hs]), hph ^ 1)) {
                    set_status(f.status, KMB_ERR_TIMEOUT_Y);
                    return false;
                }
                float2* dst = (float2*)(hand + ((size_t)(w * BS_K + hs) * 2) * 64);
                dst[lane] = make_float2(rP[0], rP[1]);
                dst[32 + lane] = make_float2(rQ[0], rQ[1]);
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&b_full[w * BS_K + hs]));
            }
            // sums over the states (fixed order) and their outputs: lane t < 3 WC reduces row
            // (j, k) = (t / 3, t % 3) for all CH channels; lane 3 WC + j reduces dlambda of column j
            __syncwarp();
            if (lane < 3 * WC) {
                const int j = lane / 3, k = lane % 3;
                if (j < ncol) {
                    const float* src = my_red + (j * 4 + k) * RS;
                    float acc[32 / MS][2];
#pragma unroll
                    for (int s2 = 0; s2 < 32 / MS; s2++) acc[s2][0] = acc[s2][1] = 0.0f;
#pragma unroll
                    for (int l = 0; l < 64; l += 4) {
                        const float4 v = *(const float4*)(src + l);
                        const int s2 = (l / 2) / MS;   // lane (l / 2) belongs to channel set s2
                        acc[s2][0] = __fadd_rn(__fadd_rn(acc[s2][0], v.x), v.z);
                        acc[s2][1] = __fadd_rn(__fadd_rn(acc[s2][1], v.y), v.w);
                    }
                    const int p = o * Q + q0 + j;
#pragma unroll
                    for (int s2 = 0; s2 < 32 / MS; s2++)
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            const int cc = 2 * s2 + c;
                            const long long pd = ((long long)b * P + p) * D + d0 + cc;
                            const float v = acc[s2][c];
                            if (G > 1) {
                                f.part[(pd * G + half) * 3 + k] = v;
                            } else if (k < 2) {
                                if (f.ddelta) {
                                    // inner axis is axis 1, outer axis 0
                                    float* dd = f.ddelta + (((long long)b * 2 + (k == 0 ? 1 : 0)) * P + p) * D + d0 + cc;
                                    *dd = OVW ? v : __fadd_rn(*dd, v);
                                }
                            } else if (f.dx) {
                                float* dd = f.dx + pd;
                                *dd = OVW ? v : __fadd_rn(*dd, v);
                            }
                        }
                }
            } else if (lane < 4 * WC) {
                const int j = lane - 3 * WC;
                if (j < ncol && f.plam) {
                    const float* src = my_red + (j * 4 + 3) * RS;
                    float acc = 0.0f;
#pragma unroll
                    for (int l = 0; l < 32; l += 4) {
                        const float4 v = *(const float4*)(src + l);
                        acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
                    }
                    f.plam[((long long)b * ngl + dt0 * G + half) * P + o * Q + q0 + j] = acc;
                }
            }
            __syncwarp();
            // rotate the state ring
#pragma unroll
            for (int j = 0; j < WC; j++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    hO[j][c] = hP[j][c];
                    bO[j][c] = bP[j][c];
                    hP[j][c] = hN[j][c];
                    bP[j][c] = bN[j][c];
                    cO[j][c] = cN[j][c];
                }
            row++;
            return true;
        };
        bool ok = true;
#pragma unroll 1
        for (int o = O - 1; o >= 1 && ok; o--) ok = do_row(std::integral_constant<bool, true>(), o);
        if (ok) ok = do_row(std::integral_constant<bool, false>(), 0);
        if (!ok) {
            cp_async_wait_all();
            return;
        }
        // per-(item, strip) partials of dA (this lane's (d, state)) and dtheta
        {
            const long long r = (long long)b * S + w;
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int d = dl0 + c;
                f.pA[((r * 2 + 1) * D + d) * M + mg] = gAI[c];
                f.pA[((r * 2 + 0) * D + d) * M + mg] = gAO[c];
            }
            if (ROPE) {
                float v = gth;
#pragma unroll
                for (int off = MS / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (ml == 0) f.pth[(((long long)b * G + half) * S + w) * (D / 2) + (dl0 >> 1)] = v;
            }
        }
    }
    cp_async_wait_all();
}

// ddelta / dx from the two state halves' partials (M = 64), fixed order.
__global__ void bwd_strips_combine(const float* __restrict__ part, float* __restrict__ ddelta, float* __restrict__ dx,
                                   long long batch, long long P, int D, int G, int overwrite) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * P * D) return;
    const long long b = i / (P * D), pd = i - b * P * D;
    float s[3] = {0.f, 0.f, 0.f};
    for (int g = 0; g < G; g++)
        for (int k = 0; k < 3; k++) s[k] = __fadd_rn(s[k], part[(i * G + g) * 3 + k]);
    if (ddelta) {
        float* d1 = ddelta + (b * 2 + 1) * P * D + pd;
        float* d0 = ddelta + (b * 2 + 0) * P * D + pd;
        *d1 = overwrite ? s[0] : __fadd_rn(*d1, s[0]);
        *d0 = overwrite ? s[1] : __fadd_rn(*d0, s[1]);
    }
    if (dx) dx[i] = overwrite ? s[2] : __fadd_rn(dx[i], s[2]);
}

// out[i] (+)= sum_j part[j * stride + i], fixed order
__global__ void bwd_strips_reduce(const float* __restrict__ part, float* __restrict__ out, long long count, long long n,
                                  long long stride, int overwrite) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float acc = 0.0f;
    for (long long j = 0; j < n; j++) acc = __fadd_rn(acc, part[j * stride + i]);
    out[i] = overwrite ? acc : __fadd_rn(out[i], acc);
}

// dlambda[b, p] (+)= sum_g plam[b, g, p], fixed order
__global__ void bwd_strips_lambda(const float* __restrict__ plam, float* __restrict__ dl, long long batch, int ngroups,
                                  long long P, int overwrite) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * P) return;
    const long long b = i / P, p = i - b * P;
    float acc = 0.0f;
    for (int g = 0; g < ngroups; g++) acc = __fadd_rn(acc, plam[(b * ngroups + g) * P + p]);
    dl[i] = overwrite ? acc : __fadd_rn(dl[i], acc);
}

// ------------------------------------------------------------------ host side
constexpr long long BS_SMAX = 8;    // most strips a grid can have (64 columns of 8)

size_t scan_bwd_strips_scratch_bytes(const ScanDesc& s) {
    const long long G = s.M == 64 ? 2 : 1;
    const long long CH = s.M == 16 ? 4 : 2;
    const long long ntd = s.D / CH;
    size_t n = 0;
    if (G > 1) n += (size_t)s.batch * s.P * s.D * G * 3;
    n += (size_t)s.batch * BS_SMAX * 2 * s.D * s.M;            // pA
    n += (size_t)s.batch * G * BS_SMAX * (s.D / 2 + 1);         // pth
    n += (size_t)s.batch * ntd * G * s.P;                       // plam
    return n * sizeof(float) + 4 * 256;
}

template <int M, bool ROPE, bool OVW, int WC>
static cudaError_t bs_launch(const BwdStripDesc& f, cudaStream_t st) {
    using Gm = BsGeom<M, WC>;
    auto k = scan_bwd_strips<M, ROPE, OVW, WC>;
    const int smem = (f.S * 3 * Gm::SMALL + f.S * Gm::ROWS * Gm::RS + f.S * BS_K * 2 * 64) * 4 + 2 * f.S * BS_K * 8;
    const int threads = f.S * 32;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev, sms, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sms = persistent_sms(sms);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, threads, smem);
    if (per < 1) return cudaErrorNotSupported;
    long long grid = (long long)sms * per;
    if (grid > f.ntiles) grid = f.ntiles;
    k<<<(unsigned)grid, threads, smem, st>>>(f);
    return cudaGetLastError();
}

template <int M, int WC>
static cudaError_t bs_dispatch(const BwdStripDesc& f, bool rope, bool ovw, cudaStream_t st) {
    if (rope) return ovw ? bs_launch<M, true, true, WC>(f, st) : bs_launch<M, true, false, WC>(f, st);
    return ovw ? bs_launch<M, false, true, WC>(f, st) : bs_launch<M, false, false, WC>(f, st);
}

// 2D grids whose inner (last) extent is <= 64, M in {16, 32, 64}, D a multiple
// of the channel tile, dB and dC given, accurate exponential.
// cudaErrorNotSupported outside that envelope.
cudaError_t launch_scan_bwd_strips(const ScanDesc& s, const float* dy, float* dA, float* dB, float* dC, float* ddelta,
                                   float* dlambda, float* dtheta, float* dx, int overwrite, void* scratch, int* status,
                                   cudaStream_t st) {
    if (s.nd != 2 || s.dims[1] > 64 || s.dims[1] < 1) return cudaErrorNotSupported;
    if (s.M != 16 && s.M != 32 && s.M != 64) return cudaErrorNotSupported;
    if (!dB || !dC || s.fast_exp) return cudaErrorNotSupported;
    const int CH = s.M == 16 ? 4 : 2;
    if (s.D % CH != 0) return cudaErrorNotSupported;
    if (s.P * s.D * s.M >= (1LL << 31)) return cudaErrorNotSupported;   // 32-bit offsets inside an item
    constexpr int WC = 8;   // measured: 4 columns per strip (16 warps, 128 registers) ran 1.6x slower
    BwdStripDesc f{};
    f.D = s.D;
    f.Q = (int)s.dims[1]; f.O = (int)s.dims[0];
    f.S = (f.Q + WC - 1) / WC;
    const int G = s.M == 64 ? 2 : 1;
    f.ntd = s.D / CH;
    f.ntiles = s.batch * f.ntd * G;
    f.has_lambda = s.has_lambda; f.clamp = s.clamp;
    f.amin = s.a_log_min; f.deflam = s.default_lambda;
    f.P = s.P;
    f.x = s.x; f.A = s.A; f.B = s.B; f.C = s.C; f.delta = s.delta; f.theta = s.theta; f.lambda = s.lambda;
    f.h = s.h; f.dy = dy;
    f.dB = dB; f.dC = dC; f.ddelta = ddelta; f.dx = dx;
    f.status = status;
    auto align = [](char* p) { return (char*)(((uintptr_t)p + 255) & ~(uintptr_t)255); };
    char* c = align((char*)scratch);
    if (G > 1) { f.part = (float*)c; c = align(c + (size_t)s.batch * s.P * s.D * G * 3 * 4); }
    f.pA = (float*)c; c = align(c + (size_t)s.batch * BS_SMAX * 2 * s.D * s.M * 4);
    f.pth = (float*)c; c = align(c + (size_t)s.batch * G * BS_SMAX * (s.D / 2 + 1) * 4);
    f.plam = dlambda ? (float*)c : nullptr;
    const bool ovw = overwrite != 0;
    cudaError_t e;
    switch (s.M) {
        case 16: e = bs_dispatch<16, WC>(f, s.rope, ovw, st); break;
        case 32: e = bs_dispatch<32, WC>(f, s.rope, ovw, st); break;
        default: e = bs_dispatch<64, WC>(f, s.rope, ovw, st); break;
    }
    if (e != cudaSuccess) return e;
    auto nb = [](long long n) { return (unsigned)((n + 255) / 256); };
    if (G > 1 && (ddelta || dx))
        bwd_strips_combine<<<nb(s.batch * s.P * s.D), 256, 0, st>>>(f.part, ddelta, dx, s.batch, s.P, s.D, G, overwrite);
    if (dA) {
        const long long cnt = 2LL * s.D * s.M;
        bwd_strips_reduce<<<nb(cnt), 256, 0, st>>>(f.pA, dA, cnt, s.batch * f.S, cnt, overwrite);
    }
    if (dtheta && s.rope && s.D >= 2) {
        const long long cnt = s.D / 2;
        bwd_strips_reduce<<<nb(cnt), 256, 0, st>>>(f.pth, dtheta, cnt, s.batch * G * f.S, s.D / 2, overwrite);
    }
    if (dlambda)
        bwd_strips_lambda<<<nb(s.batch * s.P), 256, 0, st>>>(f.plam, dlambda, s.batch, f.ntd * G, s.P, overwrite);
    return cudaGetLastError();
}

}  // namespace kmb
