// scannd_strips.cu -- Scan-A forward for 2D grids on sm_100a: a systolic
// column-strip pipeline (the headline path: 2D 64x64, D=512, M=64, batch 32).
//
// The grid is walked row by row (outer o, inner q, inner extent Q <= 64).  A
// CTA owns a tile (item b, CH consecutive channels, all M states) and splits
// the inner axis into S <= 8 column strips of Wc <= 8 columns; warp w owns
// strip w.  Each lane carries CPT = 2 channels (the RoPE pair, so the rotation
// needs no shuffle, or two independent channels) and SPT state slots (m, and
// m + 32 when M = 64): up to four independent state chains per lane, which
// amortises the per-row and per-point work and gives the scheduler ILP.  Per
// column of its strip a lane keeps the rotated state R h and the B*x product
// of the previous row in registers (ring of Wc slots).  The value left of its
// first column comes from strip w-1 through a shared-memory handoff slot
// guarded by mbarriers; strips run one row apart, like a systolic array.
// (The HW > 1 lane-half split, with y accumulated by red.add into a zeroed y,
// remains for geometries where one warp cannot cover M; the supported M of
// 16, 32 and 64 all use HW = 1.)
//
// Data: per strip a ring of NSS stages, each one row of the strip: TMA boxes
// of B and C [Wc][CH][M], x and delta [.][Wc][4] (4-channel boxes, aligned),
// lambda; issued by lane 0 of the strip's warp, NSS-1 rows ahead.  Only
// B, C, x, delta, lambda are read (once) and h, y written (once): 12 B per
// state update + 16 B per (point, channel).
// y[p, d] = sum_m C h: each lane first adds its state slots, then the warp
// reduces its 8 points x CPT channels across lanes with a transposed butterfly.
#include <cuda.h>
#include "kmb_common.cuh"
#include "kmb_sync.cuh"
#include "kmb_butterfly.cuh"
#include <type_traits>

namespace kmb {
int persistent_sms(int sms);  // SMs a persistent grid may fill (capi.cu)

// packed fp32 pairs (per component exactly __fadd_rn / __fmul_rn / __fmaf_rn)
#ifdef KMB_F2_EMUL
__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)); }
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    return make_float2(__fmaf_rn(a.x, b.x, c.x), __fmaf_rn(a.y, b.y, c.y));
}
#else
__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
#endif

constexpr int SW_NSS_MAX = 4;  // stages per strip (fewer when shared memory is short)
constexpr int SW_K = 4;        // handoff slots per strip boundary
constexpr int SW_WC = 8;       // max columns per strip

struct StripDesc {
    int D, nd;
    int Q, O, Wc, S;        // inner extent, outer extent, columns per strip, strips
    int O1;                 // 3D: rows per plane (the outer extent O is planes x O1)
    int fence_period;       // 3D: rows between proxy fences (<= O1 - look-ahead + 1)
    int k_in;               // axis of the inner dimension
    int lam_inner_fast;     // lambda box (Wc,1,1) at (q0,o,b) vs (4,Wc,1) at (o&~3,q0,b)
    int clamp;
    float amin, deflam;
    long long qstride, ostride;  // point strides of the inner / outer dims
    long long P;
    int ntd;                // channel tiles per item
    long long ntiles;
    int nss;                // stages per strip
    int st_bytes, offC, offX, offD, offL;
    unsigned tx_bytes;
    int red_y;              // 1: y is accumulated with red.add (two lane halves)
    int ex2;                // 1: alpha by one ex2.approx (opt-in), 0: expf in the reference's order
    const float* A;
    const float* theta;
    float* h;
    float* y;
    int* status;
};

template <int MT, bool ROPE>
struct StripGeom {
    // Each thread carries CPT = 2 channels (the RoPE pair, or two independent
    // channels) and, for M = 64, SPT = 2 states (m and m + 32), so one warp
    // covers a strip and the per-row and per-point work (waits, handoff, TMA
    // issue, x / delta / lambda, coefficients) serves up to four independent
    // state chains, which also gives the scheduler four-way ILP per lane.
    static constexpr int CPT = 2;                         // channels per thread
    static constexpr int SPT = MT == 64 ? 2 : 1;          // states per thread
    static constexpr int U = CPT * SPT;                   // (channel, state) units per thread
    static constexpr int SPW = MT >= 32 ? 1 : 32 / MT;    // channel sets per warp
    static constexpr int HW = MT >= 32 ? MT / (32 * SPT) : 1;  // warps per strip
    static constexpr int CH = SPW * CPT;                  // channels per tile
    static constexpr int GS = MT >= 32 ? 32 : MT;         // lanes summed for y
    static constexpr int MAXT = 8 * HW * 32;              // threads of the largest CTA (8 strips)
};

template <int MT, bool ROPE, bool P3 = false, int WCT = SW_WC>
struct StripLayout {
    using Gm = StripGeom<MT, ROPE>;
    static constexpr int BBOX = MT * Gm::CH * WCT * 4;     // bytes of one B / C box
    static constexpr int offC = BBOX;
    static constexpr int offX = 2 * BBOX;                  // x box [WC][4]
    static constexpr int offD = offX + 128;                // delta box [nd][WC][4]
    static constexpr int offL = offD + (P3 ? 384 : 256);   // lambda box [WC] or [WC][4]
    // 3D: the previous plane's h, B and x boxes (the plane predecessor of every point of the row)
    static constexpr int offHp = offL + 128;
    static constexpr int offBp = offHp + BBOX;
    static constexpr int offXp = offBp + BBOX;
    static constexpr int bytes = P3 ? offXp + 128 : offL + 128;
};

// EXPM 0: expf, reference order; 1: ex2.approx.  P3: 3D grids (planes x rows x inner, inner = the last
// axis): rows are (plane, row) pairs walked in order, the row predecessor comes from the register ring
// (none on a plane's first row) and the plane predecessor's h, B and x arrive as TMA boxes of the row
// O1 rows back, which this warp wrote itself (a proxy fence after every row orders its h stores before
// the bulk loads that read them; the issuer runs at most O1 rows ahead).
template <int MT, bool ROPE, bool LAMB, bool KIN0, bool FULL, int EXPM, bool P3 = false, int WCT = SW_WC>
__global__ void __launch_bounds__(StripGeom<MT, ROPE>::MAXT, 1)
scan_fwd_strips(const __grid_constant__ StripDesc f,
                const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mC,
                const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mD,
                const __grid_constant__ CUtensorMap mL, const __grid_constant__ CUtensorMap mH) {
    using Gm = StripGeom<MT, ROPE>;
    using Ly = StripLayout<MT, ROPE, P3, WCT>;
    constexpr bool EX2 = EXPM == 1;
    constexpr int CPT = Gm::CPT, HW = Gm::HW, CH = Gm::CH, GS = Gm::GS, U = Gm::U;
    constexpr int WC = WCT;   // columns per strip
    constexpr int ST = Ly::bytes;
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
    const int w = wi / HW, hh = wi % HW;  // strip, lane half
    // parameters held in registers
    const int S = f.S, NSS = f.nss, D = f.D, O = f.O, Q = f.Q, ntd = f.ntd;
    const long long ntiles = f.ntiles, P = f.P, qstride = f.qstride, ostride = f.ostride;
    const float deflam = f.deflam;
    const float omlq = __fmul_rn(__fsub_rn(1.0f, deflam), 0.25f);  // (1 - lambda) / 4 when lambda is constant
    const int red_y = f.red_y;
    // smem map: stages [S][NSS] | handoff values [S][HW][K][2][32*U] | barriers
    unsigned char* stages = smem;
    const int hv = 32 * U;
    float* hand = (float*)(smem + (size_t)S * NSS * ST);
    uint64_t* bars = (uint64_t*)(hand + (size_t)S * HW * SW_K * 2 * hv);
    uint64_t* b_full = bars;                          // [S][NSS]
    uint64_t* b_empty = bars + S * NSS;               // [S][NSS]
    uint64_t* b_hfull = bars + 2 * S * NSS;           // [S][HW][K]
    uint64_t* b_hempty = b_hfull + S * HW * SW_K;     // [S][HW][K]
    if (tid == 0) {
        for (int i = 0; i < S * NSS; i++) {
            mbar_init(smem_u32(&b_full[i]), 1);
            mbar_init(smem_u32(&b_empty[i]), HW);
        }
        for (int i = 0; i < S * HW * SW_K; i++) {
            mbar_init(smem_u32(&b_hfull[i]), 1);
            mbar_init(smem_u32(&b_hempty[i]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (w >= S) return;

    // ---- lane geometry
    const int m = MT >= 32 ? hh * 32 + lane : lane % MT;
    const int cl0 = MT >= 32 ? 0 : (lane / MT) * CPT;   // first local channel of this thread
    const long long DM = (long long)D * MT;
    const long long hq = qstride * DM;
    const int q0 = w * WC;
    const int ncol = FULL ? WC : min(WC, Q - q0);  // FULL: every strip has WC columns
    unsigned char* my_stages = stages + (size_t)w * NSS * ST;
    const bool issuer = (hh == 0 && lane == 0);
    const int tiles_mine = (int)((ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x);
    const int total_rows = tiles_mine * O;
    // issuer state: next row to issue, its (tile, o) and ring (slot, phase),
    // all maintained incrementally (no runtime divisions per row)
    int next_issue = 0, is_o = 0, is_slot = 0;
    uint32_t is_phase = 0;
    // issuer's tile as (item, channel tile), advanced without divisions
    int is_b = (int)(blockIdx.x / ntd), is_dt = (int)(blockIdx.x - (long long)is_b * ntd);

    auto issue = [&]() {
        const int b = is_b;
        const int d0 = is_dt * CH;
        const int o = is_o;
        unsigned char* st = my_stages + (size_t)is_slot * ST;
        const uint32_t full = smem_u32(&b_full[w * NSS + is_slot]);
        mbar_expect_tx(full, f.tx_bytes);
        tma_load_5d(smem_u32(st), &mB, full, 0, d0, q0, o, b);
        tma_load_5d(smem_u32(st + Ly::offC), &mC, full, 0, d0, q0, o, b);
        tma_load_4d(smem_u32(st + Ly::offX), &mX, full, d0 & ~3, q0, o, b);
        tma_load_5d(smem_u32(st + Ly::offD), &mD, full, d0 & ~3, q0, o, 0, b);
        if (LAMB) {
            if (!KIN0) tma_load_3d(smem_u32(st + Ly::offL), &mL, full, q0, o, b);
            else tma_load_3d(smem_u32(st + Ly::offL), &mL, full, o & ~3, q0, b);
        }
        if (P3) {   // plane predecessor row (negative rows of the first plane read zeros)
            tma_load_5d(smem_u32(st + Ly::offHp), &mH, full, 0, d0, q0, o - f.O1, b);
            tma_load_5d(smem_u32(st + Ly::offBp), &mB, full, 0, d0, q0, o - f.O1, b);
            tma_load_4d(smem_u32(st + Ly::offXp), &mX, full, d0 & ~3, q0, o - f.O1, b);
        }
    };
    auto advance_issue = [&]() {
        next_issue++;
        if (++is_o == O) {
            is_o = 0;
            for (is_dt += gridDim.x; is_dt >= ntd; is_dt -= ntd) is_b++;
        }
        if (++is_slot == NSS) { is_slot = 0; is_phase ^= 1u; }
    };
    // Keep up to NSS rows in flight; block only for the row about to be consumed.
    const int ahead = P3 ? min(NSS, f.O1) : NSS;   // P3: row r reads row r - O1, finished only when r < cur + O1
    auto top_up = [&](int cur) -> bool {
        while (next_issue < total_rows && next_issue < cur + ahead) {
            if (next_issue >= NSS) {
                // the slot's previous use (row next_issue - NSS) must have been released
                const uint32_t eb = smem_u32(&b_empty[w * NSS + is_slot]);
                const uint32_t ph = is_phase ^ 1u;
                if (next_issue <= cur) {
                    if (!mbar_wait(eb, ph)) return false;
                } else if (!mbar_try(eb, ph)) {
                    break;
                }
            }
            issue();
            advance_issue();
        }
        return true;
    };
    auto drain = [&]() {
        if (!issuer) return;
        for (int j = (next_issue > NSS ? next_issue - NSS : 0); j < next_issue; j++)
            mbar_wait(smem_u32(&b_full[w * NSS + j % NSS]), (uint32_t)((j / NSS) & 1));
    };

    float* my_hand_in = hand + ((size_t)(w * HW + hh) * SW_K) * 2 * hv;           // written by strip w-1
    float* my_hand_out = hand + ((size_t)((w + 1) * HW + hh) * SW_K) * 2 * hv;    // read by strip w+1
    const int hl = lane * U;
    // per-thread offsets inside a stage
    const int bofs = (cl0 * MT + m) * 4;                 // B / C box: [j][CH][MT]
    const int xofs = cl0;                                // x / delta box column (+ (d0 & 3))
    // y: after the butterfly, lane gl of a GS-lane group holds the sum of value
    // index butterfly_index(gl) = (column j, channel c); fixed per lane
    bool y_lane;
    long long y_col;
    {
        constexpr int NV = WC * CPT, LPV = GS / NV;
        const int gl = lane & (GS - 1);
        const int idx = butterfly_index<NV, GS>(gl);
        const int j = idx / CPT, c = idx % CPT;
        y_lane = (LPV <= 1 || (gl % LPV) == 0) && j < ncol;
        y_col = (long long)(q0 + j) * qstride * D + cl0 + c;
    }
    const long long h_ostep = ostride * DM, y_ostep = ostride * D;  // one outer step in h / y
    int row = 0, slot = 0;  // consumer row counter and its stage slot / phase
    uint32_t ph = 0;

    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int b = (int)(tile / ntd);
        const int d0 = (int)(tile - (long long)b * ntd) * CH;
        float AI[U], AO[U], AP[U], cth = 1.0f, sth = 0.0f;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int d = d0 + cl0 + u % CPT, mu = m + 32 * (u / CPT);
            // EX2: A log2 e, so alpha = 2^(delta * A log2 e) is one multiply and one ex2
            // per update; otherwise A itself and alpha = expf(delta * A) as the reference
            const float sc = EX2 ? kKmbLog2e : 1.0f;
            const int axI = P3 ? 2 : (KIN0 ? 0 : 1), axO = P3 ? 1 : (KIN0 ? 1 : 0);
            AI[u] = __fmul_rn(kmb_clampA(f.A[((long long)axI * D + d) * MT + mu], f.clamp, f.amin), sc);
            AO[u] = __fmul_rn(kmb_clampA(f.A[((long long)axO * D + d) * MT + mu], f.clamp, f.amin), sc);
            AP[u] = P3 ? __fmul_rn(kmb_clampA(f.A[(long long)d * MT + mu], f.clamp, f.amin), sc) : 0.0f;
        }
        if (ROPE) {
            const float th = f.theta[(d0 + cl0) >> 1];
            kmb_cos_sin(th, &cth, &sth);
        }
        // h and y of the current row, advanced by one outer step per row
        float* hrow = f.h + (long long)b * P * DM + (long long)(d0 + cl0) * MT + m + (long long)q0 * hq;
        float* yrow = f.y + (long long)b * P * D + d0 + y_col;
        const int xo = (d0 & 3) + xofs;
        float ring_h[WC][U], ring_b[WC][U];

        // one row of this strip; HASO: the row above exists; HASP (3D): the plane before exists
        auto do_row = [&](auto hasO_c, auto hasP_c, int o) -> bool {
            constexpr bool HASO = decltype(hasO_c)::value;
            constexpr bool HASP = decltype(hasP_c)::value;
            if (issuer && !top_up(row)) {
                set_status(f.status, KMB_ERR_TIMEOUT_EMPTY);
                drain();
                return false;
            }
            __syncwarp();
            if (!mbar_wait(smem_u32(&b_full[w * NSS + slot]), ph)) {
                set_status(f.status, KMB_ERR_TIMEOUT_FULL);
                drain();
                return false;
            }
            const unsigned char* st = my_stages + (size_t)slot * ST;
            const float* Bs = (const float*)(st + bofs);
            const float* Cs = (const float*)(st + Ly::offC + bofs);
            const float* Xs = (const float*)(st + Ly::offX) + xo;
            const float* DsI = (const float*)(st + Ly::offD) + (P3 ? 2 * WC * 4 : KIN0 ? 0 : WC * 4) + xo;
            const float* DsO = (const float*)(st + Ly::offD) + (P3 ? WC * 4 : KIN0 ? WC * 4 : 0) + xo;
            const float* DsP = (const float*)(st + Ly::offD) + xo;
            const float* Hp = (const float*)(st + Ly::offHp + bofs);
            const float* Bp = (const float*)(st + Ly::offBp + bofs);
            const float* Xp = (const float*)(st + Ly::offXp) + xo;
            const float* Ls = (const float*)(st + Ly::offL) + (KIN0 ? (o & 3) : 0);
            const int hs = row & (SW_K - 1);
            const uint32_t hph = (uint32_t)((row / SW_K) & 1);
            float lh[U], lb[U];
            if (w > 0) {
                if (!mbar_wait(smem_u32(&b_hfull[(w * HW + hh) * SW_K + hs]), hph)) {
                    set_status(f.status, KMB_ERR_TIMEOUT_Y);
                    drain();
                    return false;
                }
                const float* src = my_hand_in + (size_t)hs * 2 * hv;
#pragma unroll
                for (int u = 0; u < U; u++) {
                    lh[u] = src[hl + u];
                    lb[u] = src[hv + hl + u];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&b_hempty[(w * HW + hh) * SW_K + hs]));
            }
            float prod[WC][CPT];
            float lastH[U], lastB[U];
            float* hp = hrow;
#pragma unroll
            for (int j = 0; j < WC; j++) {
                const float lam = LAMB ? Ls[j * (KIN0 ? 4 : 1)] : deflam;
                float hn[U];
                if constexpr (!EX2) {
                    // The lane's two channels as one float2 (.x = channel cl0, .y = cl0 + 1): the
                    // reference-order operations of the scalar path below, two per packed
                    // instruction (same IEEE rounding per component); expf stays per channel.
                    const float2 x2 = *reinterpret_cast<const float2*>(Xs + j * 4);
                    const float2 dI2 = *reinterpret_cast<const float2*>(DsI + j * 4);
                    const float2 dO2 = *reinterpret_cast<const float2*>(DsO + j * 4);
                    // dt: the deltas summed in axis order (2D: inner + outer, commutative; 3D: plane, row, inner)
                    const float2 dP2 = P3 ? *reinterpret_cast<const float2*>(DsP + j * 4) : make_float2(0.0f, 0.0f);
                    const float2 dt2 = P3 ? f2add(f2add(dP2, dO2), dI2) : f2add(dI2, dO2);
                    const float2 omdt2 = f2mul(f2add(make_float2(1.0f, 1.0f), make_float2(-lam, -lam)), dt2);
                    const float2 gam2 = f2mul(make_float2(lam, lam), dt2);
#pragma unroll
                    for (int sl = 0; sl < Gm::SPT; sl++) {
                        const int u0 = sl * CPT, sofs = 32 * sl;
                        const float2 bu2 = f2mul(make_float2(Bs[j * CH * MT + sofs], Bs[j * CH * MT + MT + sofs]), x2);
                        const float2 zI = f2mul(dI2, make_float2(AI[u0], AI[u0 + 1]));
                        const float2 aI2 = make_float2(expf(zI.x), expf(zI.y));
                        const float2 hatI2 = (j == 0) ? make_float2(lh[u0], lh[u0 + 1])
                                                      : make_float2(ring_h[j == 0 ? 0 : j - 1][u0], ring_h[j == 0 ? 0 : j - 1][u0 + 1]);
                        const float2 buI2 = (j == 0) ? make_float2(lb[u0], lb[u0 + 1])
                                                     : make_float2(ring_b[j == 0 ? 0 : j - 1][u0], ring_b[j == 0 ? 0 : j - 1][u0 + 1]);
                        const float2 rh2 = make_float2(ring_h[j][u0], ring_h[j][u0 + 1]);
                        const float2 rb2 = make_float2(ring_b[j][u0], ring_b[j][u0 + 1]);
                        float2 buacc2, dacc2, hacc2;
                        float inv;
                        if constexpr (P3) {
                            // three axes in axis order (plane, row, inner); means as sum / n, n = 3 an
                            // IEEE division; hn as in the scalar 3D path
                            int n = 0;
                            buacc2 = dacc2 = hacc2 = make_float2(0.0f, 0.0f);
                            if (HASP) {
                                const float2 zP = f2mul(dP2, make_float2(AP[u0], AP[u0 + 1]));
                                const float2 aP2 = make_float2(expf(zP.x), expf(zP.y));
                                const float* hb = Hp + j * CH * MT + sofs;
                                float2 hatP2 = make_float2(hb[0], hb[MT]);
                                if (ROPE) {
                                    const float2 m = f2mul(make_float2(sth, cth), make_float2(hatP2.y, hatP2.y));
                                    hatP2 = f2fma(make_float2(cth, sth), make_float2(hatP2.x, hatP2.x), make_float2(-m.x, m.y));
                                }
                                buacc2 = f2mul(make_float2(Bp[j * CH * MT + sofs], Bp[j * CH * MT + MT + sofs]),
                                               make_float2(Xp[j * 4], Xp[j * 4 + 1]));
                                dacc2 = aP2;
                                hacc2 = f2mul(aP2, hatP2);
                                n = 1;
                            }
                            if (HASO) {
                                const float2 zO = f2mul(dO2, make_float2(AO[u0], AO[u0 + 1]));
                                const float2 aO2 = make_float2(expf(zO.x), expf(zO.y));
                                if (n == 0) {
                                    buacc2 = rb2; dacc2 = aO2; hacc2 = f2mul(aO2, rh2);
                                } else {
                                    buacc2 = f2add(buacc2, rb2);
                                    dacc2 = f2add(dacc2, aO2);
                                    hacc2 = f2fma(aO2, rh2, hacc2);
                                }
                                n++;
                            }
                            if (j > 0 || w > 0) {
                                if (n == 0) {
                                    buacc2 = buI2; dacc2 = aI2; hacc2 = f2mul(aI2, hatI2);
                                } else {
                                    buacc2 = f2add(buacc2, buI2);
                                    dacc2 = f2add(dacc2, aI2);
                                    hacc2 = f2fma(aI2, hatI2, hacc2);
                                }
                                n++;
                            }
                            const float2 buavg = n == 3 ? make_float2(__fdiv_rn(buacc2.x, 3.0f), __fdiv_rn(buacc2.y, 3.0f))
                                               : n == 2 ? f2mul(buacc2, make_float2(0.5f, 0.5f)) : buacc2;
                            const float2 alavg = n == 3 ? make_float2(__fdiv_rn(dacc2.x, 3.0f), __fdiv_rn(dacc2.y, 3.0f))
                                               : n == 2 ? f2mul(dacc2, make_float2(0.5f, 0.5f)) : dacc2;
                            const float2 hn3 = f2add(f2fma(buavg, f2mul(omdt2, alavg), f2mul(bu2, gam2)), hacc2);
                            buacc2 = hn3;   // carried to the stores below
                            inv = -1.0f;
                        } else if (HASO) {
                            const float2 zO = f2mul(dO2, make_float2(AO[u0], AO[u0 + 1]));
                            const float2 aO2 = make_float2(expf(zO.x), expf(zO.y));
                            if (j > 0 || w > 0) {
                                buacc2 = KIN0 ? f2add(buI2, rb2) : f2add(rb2, buI2);
                                dacc2 = KIN0 ? f2add(aI2, aO2) : f2add(aO2, aI2);
                                hacc2 = KIN0 ? f2fma(aO2, rh2, f2mul(aI2, hatI2))
                                             : f2fma(aI2, hatI2, f2mul(aO2, rh2));
                                inv = 0.5f;
                            } else {
                                buacc2 = rb2;
                                dacc2 = aO2;
                                hacc2 = f2mul(aO2, rh2);
                                inv = 1.0f;
                            }
                        } else if (j > 0 || w > 0) {
                            buacc2 = buI2;
                            dacc2 = aI2;
                            hacc2 = f2mul(aI2, hatI2);
                            inv = 1.0f;
                        } else {
                            buacc2 = dacc2 = hacc2 = make_float2(0.0f, 0.0f);
                            inv = 0.0f;
                        }
                        const float2 inv2 = make_float2(inv, inv);
                        const float2 hn2 = P3 ? buacc2
                                              : f2add(f2fma(f2mul(buacc2, inv2), f2mul(omdt2, f2mul(dacc2, inv2)),
                                                            f2mul(bu2, gam2)), hacc2);
                        hn[u0] = hn2.x;
                        hn[u0 + 1] = hn2.y;
                        ring_b[j][u0] = bu2.x;
                        ring_b[j][u0 + 1] = bu2.y;
                        if (j < ncol) {
                            if (P3) {   // read back by the next plane (keep in L2)
                                hp[sofs] = hn2.x;
                                hp[MT + sofs] = hn2.y;
                            } else {
                                __stcs(hp + sofs, hn2.x);
                                __stcs(hp + MT + sofs, hn2.y);
                            }
                        }
                        const float2 cy2 = f2mul(make_float2(Cs[j * CH * MT + sofs], Cs[j * CH * MT + MT + sofs]), hn2);
                        prod[j][0] = sl == 0 ? cy2.x : __fadd_rn(prod[j][0], cy2.x);
                        prod[j][1] = sl == 0 ? cy2.y : __fadd_rn(prod[j][1], cy2.y);
                    }
                } else {
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = u % CPT, sofs = 32 * (u / CPT);  // channel, state offset
                    const float x = Xs[j * 4 + c];
                    const float dI = DsI[j * 4 + c];
                    const float dO = DsO[j * 4 + c];
                    const float Bv = Bs[j * CH * MT + c * MT + sofs];
                    const float dt = __fadd_rn(dI, dO);
                    const float bu = __fmul_rn(Bv, x);
                    const float aI = EX2 ? kmb_ex2(__fmul_rn(dI, AI[u])) : expf(__fmul_rn(dI, AI[u]));
                    float buacc, dacc, hacc, inv;
                    // inner predecessor: the previous column (strip w-1's last column when j == 0)
                    const float hatI = (j == 0) ? lh[u] : ring_h[j == 0 ? 0 : j - 1][u];
                    const float buI = (j == 0) ? lb[u] : ring_b[j == 0 ? 0 : j - 1][u];
                    if constexpr (P3) {
                        // reference order over the axes (plane, row, inner): dt = sum of the three
                        // deltas; sums of the present predecessors' Bu, alpha and alpha * h in axis
                        // order; means as sum / n (n = 3 an IEEE division)
                        const float dP = DsP[j * 4 + c];
                        const float dt3 = __fadd_rn(__fadd_rn(dP, dO), dI);
                        int n = 0;
                        buacc = 0.0f; dacc = 0.0f; hacc = 0.0f;
                        if (HASP) {
                            const float aP = expf(__fmul_rn(dP, AP[u]));
                            const float* hb = Hp + j * CH * MT + sofs;
                            float hatP;
                            if (ROPE) {
                                const float h0 = hb[0], h1 = hb[MT];
                                hatP = c == 0 ? __fmaf_rn(cth, h0, -__fmul_rn(sth, h1))
                                              : __fmaf_rn(sth, h0, __fmul_rn(cth, h1));
                            } else {
                                hatP = hb[c * MT];
                            }
                            buacc = __fmul_rn(Bp[j * CH * MT + c * MT + sofs], Xp[j * 4 + c]);
                            dacc = aP;
                            hacc = __fmul_rn(aP, hatP);
                            n = 1;
                        }
                        if (HASO) {
                            const float aO = expf(__fmul_rn(dO, AO[u]));
                            if (n == 0) {
                                buacc = ring_b[j][u]; dacc = aO; hacc = __fmul_rn(aO, ring_h[j][u]);
                            } else {
                                buacc = __fadd_rn(buacc, ring_b[j][u]);
                                dacc = __fadd_rn(dacc, aO);
                                hacc = __fmaf_rn(aO, ring_h[j][u], hacc);
                            }
                            n++;
                        }
                        if (j > 0 || w > 0) {
                            if (n == 0) {
                                buacc = buI; dacc = aI; hacc = __fmul_rn(aI, hatI);
                            } else {
                                buacc = __fadd_rn(buacc, buI);
                                dacc = __fadd_rn(dacc, aI);
                                hacc = __fmaf_rn(aI, hatI, hacc);
                            }
                            n++;
                        }
                        const float buavg = n == 3 ? __fdiv_rn(buacc, 3.0f) : n == 2 ? __fmul_rn(buacc, 0.5f) : buacc;
                        const float alavg = n == 3 ? __fdiv_rn(dacc, 3.0f) : n == 2 ? __fmul_rn(dacc, 0.5f) : dacc;
                        const float beta = __fmul_rn(__fmul_rn(__fsub_rn(1.0f, lam), dt3), alavg);
                        const float gamma = __fmul_rn(lam, dt3);
                        hn[u] = __fadd_rn(__fmaf_rn(buavg, beta, __fmul_rn(bu, gamma)), hacc);
                        goto have_h;
                    }
                    if (HASO) {
                        const float aO = EX2 ? kmb_ex2(__fmul_rn(dO, AO[u])) : expf(__fmul_rn(dO, AO[u]));
                        if (!EX2 && (j > 0 || w > 0)) {
                            // reference order (src/scan_nd.c:141-168): sums over the axes in
                            // axis order, means as sum * 1/2 (exact), beta = ((1-lam) dt) mean(alpha)
                            buacc = __fadd_rn(KIN0 ? buI : ring_b[j][u], KIN0 ? ring_b[j][u] : buI);
                            dacc = __fadd_rn(KIN0 ? aI : aO, KIN0 ? aO : aI);
                            hacc = KIN0 ? __fmaf_rn(aO, ring_h[j][u], __fmul_rn(aI, hatI))
                                        : __fmaf_rn(aI, hatI, __fmul_rn(aO, ring_h[j][u]));
                            inv = 0.5f;
                        } else if (j > 0 || w > 0) {
                            // two predecessors: mean of two = sum * 0.5 (exact), so the
                            // coefficient (1-lam) dt (dacc/2) (buacc/2) is ((1-lam) dt / 4) (dacc buacc);
                            // h = (A-part + that) + gamma bu, as two fused multiply-adds
                            buacc = __fadd_rn(buI, ring_b[j][u]);
                            dacc = __fadd_rn(aI, aO);
                            hacc = KIN0 ? __fmaf_rn(aO, ring_h[j][u], __fmul_rn(aI, hatI))
                                        : __fmaf_rn(aI, hatI, __fmul_rn(aO, ring_h[j][u]));
                            const float omdtq = LAMB ? __fmul_rn(__fmul_rn(__fsub_rn(1.0f, lam), dt), 0.25f)
                                                     : __fmul_rn(omlq, dt);
                            const float gamma2 = __fmul_rn(lam, dt);
                            hn[u] = __fmaf_rn(gamma2, bu, __fmaf_rn(omdtq, __fmul_rn(dacc, buacc), hacc));
                            goto have_h;
                        } else {
                            buacc = ring_b[j][u];
                            dacc = aO;
                            hacc = __fmul_rn(aO, ring_h[j][u]);
                            inv = 1.0f;
                        }
                    } else {
                        if (j > 0 || w > 0) {
                            buacc = buI;
                            dacc = aI;
                            hacc = __fmul_rn(aI, hatI);
                            inv = 1.0f;
                        } else {
                            buacc = 0.0f;
                            dacc = 0.0f;
                            hacc = 0.0f;
                            inv = 0.0f;
                        }
                    }
                    {
                        const float beta = __fmul_rn(__fmul_rn(__fsub_rn(1.0f, lam), dt), __fmul_rn(dacc, inv));
                        const float gamma = __fmul_rn(lam, dt);
                        hn[u] = EX2 ? __fadd_rn(__fmaf_rn(bu, gamma, __fmul_rn(__fmul_rn(buacc, inv), beta)), hacc)
                                    : __fadd_rn(__fmaf_rn(__fmul_rn(buacc, inv), beta, __fmul_rn(bu, gamma)), hacc);
                    }
                have_h:
                    ring_b[j][u] = bu;
                    if (j < ncol) {
                        if (P3) hp[(long long)c * MT + sofs] = hn[u];   // read back by the next plane (keep in L2)
                        else __stcs(hp + (long long)c * MT + sofs, hn[u]);
                    }
                    const float cy = __fmul_rn(Cs[j * CH * MT + c * MT + sofs], hn[u]);
                    prod[j][c] = sofs == 0 ? cy : __fadd_rn(prod[j][c], cy);
                }
                }   // scalar path
                if (ROPE) {
                    // the pair (2i, 2i+1) of state slot s is units (s CPT, s CPT + 1)
#pragma unroll
                    for (int s = 0; s < Gm::SPT; s++) {
                        const float h0 = hn[s * CPT], h1 = hn[s * CPT + 1];
                        ring_h[j][s * CPT] = __fmaf_rn(cth, h0, -__fmul_rn(sth, h1));
                        ring_h[j][s * CPT + 1] = __fmaf_rn(sth, h0, __fmul_rn(cth, h1));
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < U; u++) ring_h[j][u] = hn[u];
                }
                if (j == 0 || j < ncol) {
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        lastH[u] = ring_h[j][u];
                        lastB[u] = ring_b[j][u];
                    }
                }
                hp += hq;
            }
            // right boundary to strip w+1
            if (w + 1 < S) {
                if (row >= SW_K &&
                    !mbar_wait(smem_u32(&b_hempty[((w + 1) * HW + hh) * SW_K + hs]), hph ^ 1)) {
                    set_status(f.status, KMB_ERR_TIMEOUT_Y);
                    drain();
                    return false;
                }
                float* dst = my_hand_out + (size_t)hs * 2 * hv;
#pragma unroll
                for (int u = 0; u < U; u++) {
                    dst[hl + u] = lastH[u];
                    dst[hv + hl + u] = lastB[u];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&b_hfull[((w + 1) * HW + hh) * SW_K + hs]));
            }
            // y: reduce the warp's WC x CPT products across its GS-lane groups
            {
                constexpr int NV = WC * CPT;
                float v[NV];
#pragma unroll
                for (int j = 0; j < WC; j++)
#pragma unroll
                    for (int c = 0; c < CPT; c++) v[j * CPT + c] = prod[j][c];
                const float sum = butterfly<NV, GS>(v, lane);
                if (y_lane) {
                    if (red_y) atomicAdd(yrow, sum);
                    else *yrow = sum;
                }
            }
            // 3D: order this warp's h stores before the bulk loads that read them back O1 rows later;
            // one fence every fence_period rows covers the rows before it
            if (P3 && (row + 1) % f.fence_period == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&b_empty[w * NSS + slot]));
            row++;
            if (++slot == NSS) { slot = 0; ph ^= 1u; }
            hrow += h_ostep;
            yrow += y_ostep;
            return true;
        };

        using T_ = std::integral_constant<bool, true>;
        using F_ = std::integral_constant<bool, false>;
        if constexpr (P3) {
            const int O1 = f.O1;
            int a1 = 0;
#pragma unroll 1
            for (int o = 0; o < O; o++) {
                bool ok;
                if (o < O1) ok = a1 == 0 ? do_row(F_(), F_(), o) : do_row(T_(), F_(), o);
                else ok = a1 == 0 ? do_row(F_(), T_(), o) : do_row(T_(), T_(), o);
                if (!ok) return;
                if (++a1 == O1) a1 = 0;
            }
        } else {
            if (!do_row(F_(), F_(), 0)) return;
#pragma unroll 1
            for (int o = 1; o < O; o++)
                if (!do_row(T_(), F_(), o)) return;
        }
    }
}

// ------------------------------------------------------------------ host side
bool tmap_encode(CUtensorMap* m, const void* base, int rank, const unsigned long long* dims,
                 const unsigned long long* strides_bytes, const unsigned* box);


template <int MT, bool ROPE, bool LAMB, bool KIN0, bool P3>
static cudaError_t strips_inst(const StripDesc& f, const CUtensorMap* maps, int smem, int threads, cudaStream_t st) {
    // 3D: four-column strips when the inner extent is <= 32, so up to eight strips (warps) share the SM
    auto k = P3 ? (f.Wc == 4 ? ((f.Q % 4 == 0) ? scan_fwd_strips<MT, ROPE, LAMB, false, true, 0, P3, 4>
                                               : scan_fwd_strips<MT, ROPE, LAMB, false, false, 0, P3, 4>)
                             : ((f.Q % SW_WC == 0) ? scan_fwd_strips<MT, ROPE, LAMB, false, true, 0, P3, SW_WC>
                                                   : scan_fwd_strips<MT, ROPE, LAMB, false, false, 0, P3, SW_WC>))
         : f.ex2 == 1 ? ((f.Q % SW_WC == 0) ? scan_fwd_strips<MT, ROPE, LAMB, KIN0, true, 1>
                                            : scan_fwd_strips<MT, ROPE, LAMB, KIN0, false, 1>)
                      : ((f.Q % SW_WC == 0) ? scan_fwd_strips<MT, ROPE, LAMB, KIN0, true, 0>
                                            : scan_fwd_strips<MT, ROPE, LAMB, KIN0, false, 0>);
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
    k<<<(unsigned)grid, threads, smem, st>>>(f, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5]);
    return cudaGetLastError();
}

template <int MT, bool ROPE>
static cudaError_t strips_flags(const ScanDesc& s, const StripDesc& f, const CUtensorMap* maps, int smem,
                                int threads, cudaStream_t st) {
    if (f.nd == 3)
        return s.has_lambda ? strips_inst<MT, ROPE, true, false, true>(f, maps, smem, threads, st)
                            : strips_inst<MT, ROPE, false, false, true>(f, maps, smem, threads, st);
    const bool k0 = f.k_in == 0;
    if (s.has_lambda)
        return k0 ? strips_inst<MT, ROPE, true, true, false>(f, maps, smem, threads, st)
                  : strips_inst<MT, ROPE, true, false, false>(f, maps, smem, threads, st);
    return k0 ? strips_inst<MT, ROPE, false, true, false>(f, maps, smem, threads, st)
              : strips_inst<MT, ROPE, false, false, false>(f, maps, smem, threads, st);
}

template <int MT, bool ROPE>
static cudaError_t strips_launch(const ScanDesc& s, int* status, cudaStream_t st) {
    using Gm = StripGeom<MT, ROPE>;
    const int CH = Gm::CH, HW = Gm::HW;
    const int D = s.D;
    if (D % CH != 0) return cudaErrorNotSupported;
    const bool p3 = s.nd == 3;
    const long long H = p3 ? s.dims[0] * s.dims[1] : s.dims[0], W = p3 ? s.dims[2] : s.dims[1];
    StripDesc f{};
    f.D = D;
    f.nd = s.nd;
    f.O1 = p3 ? (int)s.dims[1] : 1;
    if (p3) {
        // inner axis = the last one; rows = (plane, row) pairs
        if (W > 64 || H > 0x7fffffffLL) return cudaErrorNotSupported;
        f.Q = (int)W; f.O = (int)H; f.k_in = 2; f.qstride = 1; f.ostride = W; f.lam_inner_fast = 1;
    } else if (W <= 64) {
        f.Q = (int)W; f.O = (int)H; f.k_in = 1; f.qstride = 1; f.ostride = W; f.lam_inner_fast = 1;
    } else if (H <= 64) {
        f.Q = (int)H; f.O = (int)W; f.k_in = 0; f.qstride = W; f.ostride = 1; f.lam_inner_fast = 0;
    } else {
        return cudaErrorNotSupported;
    }
    if (s.has_lambda && (W % 4) != 0) return cudaErrorNotSupported;
    f.Wc = (p3 && W <= 32) ? 4 : SW_WC;
    f.S = (f.Q + f.Wc - 1) / f.Wc;
    f.clamp = s.clamp; f.amin = s.a_log_min; f.deflam = s.default_lambda;
    f.P = s.P;
    f.ntd = D / CH;
    f.ntiles = s.batch * f.ntd;
    using Ly = StripLayout<MT, ROPE>;
    using Ly3 = StripLayout<MT, ROPE, true>;
    using Ly34 = StripLayout<MT, ROPE, true, 4>;
    const int bbox = Ly::BBOX / SW_WC * f.Wc;   // B / C box bytes at this strip width
    f.offC = Ly::offC;
    f.offX = Ly::offX;
    f.offD = p3 ? Ly3::offD : Ly::offD;
    f.offL = p3 ? Ly3::offL : Ly::offL;
    f.st_bytes = p3 ? (f.Wc == 4 ? Ly34::bytes : Ly3::bytes) : Ly::bytes;
    f.tx_bytes = (unsigned)(2 * bbox + 16 * f.Wc + s.nd * 16 * f.Wc +
                            (s.has_lambda ? (f.lam_inner_fast ? 4 * f.Wc : 16 * f.Wc) : 0) +
                            (p3 ? 2 * bbox + 16 * f.Wc : 0));
    f.red_y = HW > 1;
    f.ex2 = s.ex2;
    f.A = s.A; f.theta = s.theta; f.h = s.h; f.y = s.y; f.status = status;
    const unsigned long long P = s.P, Bn = s.batch, DM = (unsigned long long)D * MT;
    const unsigned long long qs = f.qstride, os = f.ostride;
    CUtensorMap maps[6];
    memset(maps, 0, sizeof(maps));
    {
        const unsigned long long dims[5] = {(unsigned long long)MT, (unsigned long long)D, (unsigned long long)f.Q,
                                            (unsigned long long)f.O, Bn};
        const unsigned long long str[4] = {(unsigned long long)MT * 4, qs * DM * 4, os * DM * 4, P * DM * 4};
        const unsigned box[5] = {(unsigned)MT, (unsigned)CH, (unsigned)f.Wc, 1, 1};
        if (!tmap_encode(&maps[0], s.B, 5, dims, str, box)) return cudaErrorNotSupported;
        if (!tmap_encode(&maps[1], s.C, 5, dims, str, box)) return cudaErrorNotSupported;
        if (p3 && !tmap_encode(&maps[5], s.h, 5, dims, str, box)) return cudaErrorNotSupported;
    }
    {
        const unsigned long long dims[4] = {(unsigned long long)D, (unsigned long long)f.Q, (unsigned long long)f.O, Bn};
        const unsigned long long str[3] = {qs * D * 4, os * D * 4, P * D * 4};
        const unsigned box[4] = {4, (unsigned)f.Wc, 1, 1};
        if (!tmap_encode(&maps[2], s.x, 4, dims, str, box)) return cudaErrorNotSupported;
    }
    {
        const unsigned long long nd = (unsigned long long)s.nd;
        const unsigned long long dims[5] = {(unsigned long long)D, (unsigned long long)f.Q, (unsigned long long)f.O, nd, Bn};
        const unsigned long long str[4] = {qs * D * 4, os * D * 4, P * D * 4, nd * P * D * 4};
        const unsigned box[5] = {4, (unsigned)f.Wc, 1, (unsigned)nd, 1};
        if (!tmap_encode(&maps[3], s.delta, 5, dims, str, box)) return cudaErrorNotSupported;
    }
    if (s.has_lambda) {   // [H][W] per item (3D: H = planes x rows)
        const unsigned long long dims[3] = {(unsigned long long)W, (unsigned long long)H, Bn};
        const unsigned long long str[2] = {(unsigned long long)W * 4, P * 4};
        const unsigned box[3] = {f.lam_inner_fast ? (unsigned)f.Wc : 4u, f.lam_inner_fast ? 1u : (unsigned)f.Wc, 1};
        if (!tmap_encode(&maps[4], s.lambda, 3, dims, str, box)) return cudaErrorNotSupported;
    } else {
        maps[4] = maps[2];
    }
    if (!p3) maps[5] = maps[0];
    const int threads = f.S * HW * 32;
    const int hv = 32 * Gm::U;
    const int fixed = f.S * HW * SW_K * 2 * hv * 4 + (2 * f.S * SW_NSS_MAX + 2 * f.S * HW * SW_K) * 8;
    f.nss = SW_NSS_MAX;
    while (f.nss > 2 && fixed + f.S * f.nss * f.st_bytes > 227 * 1024) f.nss--;
    const int smem = fixed + f.S * f.nss * f.st_bytes;
    if (smem > 227 * 1024) return cudaErrorNotSupported;
    {
        // the issuer runs min(nss, O1) rows ahead: row r (read back at row r + O1) must be fenced before
        // the issue of row r + O1, which happens at the start of row r + O1 - ahead + 1
        const int ahead = f.nss < f.O1 ? f.nss : f.O1;
        int per = f.O1 - ahead + 1;
        if (per > 16) per = 16;
        if (per < 1) per = 1;
        f.fence_period = per;
    }
    if (f.red_y) {
        cudaError_t e = cudaMemsetAsync(s.y, 0, (size_t)s.batch * s.P * D * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    return strips_flags<MT, ROPE>(s, f, maps, smem, threads, st);
}

// 2D grids with an inner extent <= 64 and 3D grids whose last extent is <= 64 (reference-order expf
// only), M in {16, 32, 64}.
cudaError_t launch_scan_fwd_strips(const ScanDesc& s, int* status, cudaStream_t st) {
    if ((s.nd != 2 && s.nd != 3) || s.fast_exp || (s.nd == 3 && s.ex2)) return cudaErrorNotSupported;
    if (s.batch > 0x7fffffff || s.P > 0x7fffffffLL) return cudaErrorNotSupported;
    if (s.D % 4 != 0) return cudaErrorNotSupported;
    switch (s.M) {
        case 16: return s.rope ? strips_launch<16, true>(s, status, st) : strips_launch<16, false>(s, status, st);
        case 32: return s.rope ? strips_launch<32, true>(s, status, st) : strips_launch<32, false>(s, status, st);
        case 64: return s.rope ? strips_launch<64, true>(s, status, st) : strips_launch<64, false>(s, status, st);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace kmb
