// blockscan.cu -- Mamba-3 block scan (Scan-B) forward and exact backward.
//
// Reference: src/mamba_block.c:384-470 (forward, 1D and ND) and the exact
// adjoint of it (the reference's ND backward, :572-696, averages predecessors).
// One CTA owns one batch item and walks the wavefront levels of its grid
// (level = sum of coordinates; the level lists come from the host wavefront
// plan, uploaded once per shape).  Inside a level every warp takes one grid
// point; lane p owns the RoPE state pair (2p, 2p+1), so the rotation needs no
// data exchange, and the reductions over states (y = sum_n C h, and in the
// backward du, ddt, dlambda) are warp shuffles.  Predecessor states written in
// the previous level are read back from global memory after __syncthreads.
// The backward stores every point's state adjoint g_h in a scratch array and
// pulls its successors' values (no atomics); dA_log and dtheta are reduced
// from per-item partials in a fixed order.
#include <cuda_bf16.h>
#include "kmb_common.cuh"
#include "kmb_sync.cuh"
#include "kmb_butterfly.cuh"
#include "../../include/kmamba_block.h"

namespace kmb {

constexpr int BS_MAXND = 8;

__device__ __forceinline__ float ldv(const float* p) { return *p; }
__device__ __forceinline__ float ldv(const __nv_bfloat16* p) { return __bfloat162float(*p); }

struct BSDesc {
    int nd, N, R, P2, fast, bf16;
    int GP, NG;             // pairs per group, groups (CTAs per item)
    float deflam;
    long long L, batch;
    int dims[BS_MAXND], strides[BS_MAXND];
    int nlev;
    const int* lev_start;   // [nlev + 1]
    const int* lev_pts;     // [L]
    const int* lev_pos;     // [L] position of a point inside its level
    const int* nbr;         // [L] bit k: predecessor along k, bit 8 + k: successor along k
    int wmax;               // widest level
    const void *u, *dt, *lam, *B, *C;  // float, or __nv_bfloat16 when bf16
    const float *A, *theta;
    float *h, *Bu, *y;
    float* part;            // NG > 1: per-group partials of y [NG][batch][L][R]
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void bs_unravel(const BSDesc& s, int t, int* idx) {
    for (int k = 0; k < s.nd; k++) idx[k] = (t / s.strides[k]) % s.dims[k];
}

// Lane geometry shared by the forward and the backward.  The state pairs are
// split into NG groups of GP pairs; CTA (item b, group g) owns group g of item
// b, and a warp works on PPW = 32 / GP points of a level at once: lane =
// (point slot ps, pair pl).  Sums over the states of a point are shuffles
// inside the GP-lane group; with NG > 1 each group writes its partial of
// every such sum to scratch and bs_group_reduce adds the NG partials in group
// order (deterministic).
template <int GP>
struct BSLanes {
    static constexpr int PPW = 32 / GP;
    int b, g, ps, pl, n0, n1;
    bool h0ok, h1ok, pair;
    __device__ BSLanes(const BSDesc& s) {
        b = blockIdx.x / s.NG;
        g = blockIdx.x - b * s.NG;
        const int lane = threadIdx.x & 31;
        ps = lane / GP;
        pl = lane % GP;
        const int p = g * GP + pl;
        n0 = 2 * p;
        n1 = 2 * p + 1;
        h0ok = n0 < s.N;
        h1ok = n1 < s.N;
        pair = h1ok;
    }
};

template <int GP>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = GP / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Per-point inputs of the forward that do not depend on the recurrence (RM >= R
// ranks held; RM = 0: loaded at use).  A lane loads the next point's set while
// it computes the current one, across the level barrier, so the level loop
// waits only on the predecessor states.
template <int RM>
struct BSIn {
    static constexpr int K = RM > 0 ? RM : 1;
    int t;
    bool act;
    float dt, lam, u[K], b0[K], b1[K], c0[K], c1[K];
};

template <typename T, int GP, int RM>
__global__ void __launch_bounds__(512) blockscan_fwd_kernel(BSDesc s) {
    using Ln = BSLanes<GP>;
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0, n1 = ln.n1;
    const bool h0ok = ln.h0ok, h1ok = ln.h1ok, pair = ln.pair;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR;
    float* h = s.h + b * L * N;
    float* Bu = s.Bu + b * L * N;
    // y, or this group's partial of y
    float* y = (s.NG == 1 ? s.y : s.part + (long long)ln.g * s.batch * L * R) + b * L * R;
    const int step = nw * Ln::PPW;
    auto load = [&](int lvl, int base, BSIn<RM>& d) {
        d.act = base + ln.ps < s.lev_start[lvl + 1];
        const int t = s.lev_pts[d.act ? base + ln.ps : base];
        d.t = t;
        d.dt = ldv(dtp + t);
        d.lam = lamp ? ldv(lamp + t) : s.deflam;
        if constexpr (RM > 0) {
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r < R) {
                    const int c = t * NR + r * N;
                    d.u[r] = ldv(u + t * R + r);
                    d.b0[r] = h0ok ? ldv(Bp + c + n0) : 0.0f;
                    d.b1[r] = h1ok ? ldv(Bp + c + n1) : 0.0f;
                    d.c0[r] = h0ok ? ldv(Cp + c + n0) : 0.0f;
                    d.c1[r] = h1ok ? ldv(Cp + c + n1) : 0.0f;
                }
            }
        }
    };
    // this warp's next task: level nl, first point nb (nl == nlev: none left)
    int nl = 0, nb = s.lev_start[0] + warp * Ln::PPW;
    auto seek = [&]() {
        while (nl < s.nlev && nb >= s.lev_start[nl + 1]) {
            nl++;
            if (nl < s.nlev) nb = s.lev_start[nl] + warp * Ln::PPW;
        }
    };
    seek();
    BSIn<RM> nx;
    if (nl < s.nlev) load(nl, nb, nx);
    for (int lev = 0; lev < s.nlev; lev++) {
        while (nl == lev) {
            const BSIn<RM> cur = nx;
            nb += step;
            seek();
            if (nl < s.nlev) load(nl, nb, nx);
            const int t = cur.t;
            const bool act = cur.act, w0 = act && h0ok, w1 = act && h1ok;
            const float dt = cur.dt, lam = cur.lam;
            float bu0 = 0.0f, bu1 = 0.0f;
            if constexpr (RM > 0) {
#pragma unroll
                for (int r = 0; r < RM; r++) {
                    if (r < R) {
                        bu0 = __fmaf_rn(cur.b0[r], cur.u[r], bu0);
                        bu1 = __fmaf_rn(cur.b1[r], cur.u[r], bu1);
                    }
                }
            } else {
                for (int r = 0; r < R; r++) {
                    const float ur = ldv(u + t * R + r);
                    if (h0ok) bu0 = __fmaf_rn(ldv(Bp + t * NR + r * N + n0), ur, bu0);
                    if (h1ok) bu1 = __fmaf_rn(ldv(Bp + t * NR + r * N + n1), ur, bu1);
                }
            }
            const float al0 = kmb_exp(dt * A0, s.fast), al1 = kmb_exp(dt * A1, s.fast);
            float hn0, hn1;
            if (s.nd >= 2) {
                int idx[BS_MAXND];
                bs_unravel(s, t, idx);
                float bacc0 = 0.0f, bacc1 = 0.0f;
                hn0 = 0.0f;
                hn1 = 0.0f;
                int np = 0;
                for (int k = 0; k < s.nd; k++) {
                    if (idx[k] == 0) continue;
                    const int q = (t - s.strides[k]) * N;
                    const float p0 = h0ok ? h[q + n0] : 0.0f, p1 = h1ok ? h[q + n1] : 0.0f;
                    const float r0 = pair ? cth * p0 - sth * p1 : p0;
                    const float r1 = sth * p0 + cth * p1;
                    hn0 = __fmaf_rn(al0, r0, hn0);
                    hn1 = __fmaf_rn(al1, r1, hn1);
                    if (h0ok) bacc0 += Bu[q + n0];
                    if (h1ok) bacc1 += Bu[q + n1];
                    np++;
                }
                if (np > 0) {
                    const float bs = (1.0f - lam) * dt / (float)np;
                    hn0 = __fmaf_rn(bs * al0, bacc0, hn0);
                    hn1 = __fmaf_rn(bs * al1, bacc1, hn1);
                }
                const float gm = lam * dt;
                hn0 = __fmaf_rn(gm, bu0, hn0);
                hn1 = __fmaf_rn(gm, bu1, hn1);
            } else {
                // 1D recurrence (reference src/mamba_block.c:384-393)
                float p0 = 0.0f, p1 = 0.0f, pb0 = 0.0f, pb1 = 0.0f;
                if (t > 0) {
                    const int q = (t - 1) * N;
                    if (h0ok) { p0 = h[q + n0]; pb0 = Bu[q + n0]; }
                    if (h1ok) { p1 = h[q + n1]; pb1 = Bu[q + n1]; }
                }
                const float r0 = pair ? cth * p0 - sth * p1 : p0;
                const float r1 = sth * p0 + cth * p1;
                const float beta0 = (1.0f - lam) * dt * al0, beta1 = (1.0f - lam) * dt * al1;
                const float gm = lam * dt;
                hn0 = __fmaf_rn(gm, bu0, __fmaf_rn(beta0, pb0, al0 * r0));
                hn1 = __fmaf_rn(gm, bu1, __fmaf_rn(beta1, pb1, al1 * r1));
            }
            const int o = t * N;
            if (w0) { h[o + n0] = hn0; Bu[o + n0] = bu0; }
            if (w1) { h[o + n1] = hn1; Bu[o + n1] = bu1; }
            auto emit_y = [&](int r, float c0v, float c1v) {
                float part = 0.0f;
                if (h0ok) part = c0v * hn0;
                if (h1ok) part = __fmaf_rn(c1v, hn1, part);
                part = group_sum<GP>(part);
                if (act && ln.pl == 0) y[t * R + r] = part;
            };
            if constexpr (RM > 0) {
#pragma unroll
                for (int r = 0; r < RM; r++)
                    if (r < R) emit_y(r, cur.c0[r], cur.c1[r]);
            } else {
                for (int r = 0; r < R; r++)
                    emit_y(r, h0ok ? ldv(Cp + t * NR + r * N + n0) : 0.0f,
                           h1ok ? ldv(Cp + t * NR + r * N + n1) : 0.0f);
            }
        }
        __syncthreads();
    }
}

// Forward for NDT <= 3 dimensions, R <= RM <= 4: the previous level's states
// and B*u products of this CTA's pairs live in a two-level shared-memory ring
// ([2][wmax][GP][2] each), so a point reads its predecessors in shared memory;
// the next point's inputs (B, C, u, dt, lambda, neighbour mask, predecessor
// positions) are prefetched into registers across the level barrier.
template <int RM, int NDT>
struct BSInR {
    int t, nb, pos, ppos[NDT];
    bool act;
    float dt, lam, u[RM], b0[RM], b1[RM], c0[RM], c1[RM];
};

template <typename T, int GP, int RM, int NDT>
__global__ void __launch_bounds__(512) blockscan_fwd_ring(BSDesc s) {
    using Ln = BSLanes<GP>;
    extern __shared__ float bs_ring[];
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0, n1 = ln.n1, pl = ln.pl;
    const bool h0ok = ln.h0ok, h1ok = ln.h1ok, pair = ln.pair;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R, wmax = s.wmax;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    int strides[NDT];
#pragma unroll
    for (int k = 0; k < NDT; k++) strides[k] = NDT == 1 ? 1 : s.strides[k];
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR;
    float* h = s.h + b * L * N;
    float* Bu = s.Bu + b * L * N;
    float* y = (s.NG == 1 ? s.y : s.part + (long long)ln.g * s.batch * L * R) + b * L * R;
    float* ring_h = bs_ring;                          // [2][wmax][GP][2]
    float* ring_b = bs_ring + 2 * (size_t)wmax * GP * 2;
    auto rix = [&](int buf, int pos) { return ((buf * wmax + pos) * GP + pl) * 2; };
    const int step = nw * Ln::PPW;
    const int Lp = (int)L;
    // Two-deep prefetch: the point id of the task after next is read one task
    // earlier than its data, so no load in the loop waits on another load.
    struct Pt {
        int t, i;
    };
    auto point_of = [&](int lvl, int base) {
        Pt q;
        q.i = base + ln.ps;
        q.t = s.lev_pts[min(q.i, Lp - 1)];
        return q;
    };
    auto load = [&](int lvl, const Pt& q, BSInR<RM, NDT>& d) {
        const int beg = s.lev_start[lvl];
        d.act = q.i < s.lev_start[lvl + 1];
        // inactive slots compute on some valid point (clamped id) and store nothing
        const int t = q.t;
        d.t = t;
        d.pos = q.i - beg;
        d.nb = s.nbr[t];
#pragma unroll
        for (int k = 0; k < NDT; k++) d.ppos[k] = (d.nb >> k) & 1 ? s.lev_pos[t - strides[k]] : 0;
        d.dt = ldv(dtp + t);
        d.lam = lamp ? ldv(lamp + t) : s.deflam;
#pragma unroll
        for (int r = 0; r < RM; r++) {
            const bool rr = r < R;
            const int c = t * NR + (rr ? r : 0) * N;
            d.u[r] = rr ? ldv(u + t * R + r) : 0.0f;
            d.b0[r] = rr && h0ok ? ldv(Bp + c + n0) : 0.0f;
            d.b1[r] = rr && h1ok ? ldv(Bp + c + n1) : 0.0f;
            d.c0[r] = rr && h0ok ? ldv(Cp + c + n0) : 0.0f;
            d.c1[r] = rr && h1ok ? ldv(Cp + c + n1) : 0.0f;
        }
    };
    auto seek = [&](int& l, int& base) {
        while (l < s.nlev && base >= s.lev_start[l + 1]) {
            l++;
            if (l < s.nlev) base = s.lev_start[l] + warp * Ln::PPW;
        }
    };
    // task k+1 (data in nx) at (nl, nbase); task k+2 (point id in p2) at (nl2, nb2)
    int nl = 0, nbase = s.lev_start[0] + warp * Ln::PPW;
    seek(nl, nbase);
    BSInR<RM, NDT> nx;
    if (nl < s.nlev) load(nl, point_of(nl, nbase), nx);
    int nl2 = nl, nb2 = nbase + step;
    seek(nl2, nb2);
    Pt p2 = nl2 < s.nlev ? point_of(nl2, nb2) : Pt{0, 0};
    for (int lev = 0; lev < s.nlev; lev++) {
        const int cb = lev & 1, pb = cb ^ 1;
        while (nl == lev) {
            const BSInR<RM, NDT> cur = nx;
            nl = nl2;
            nbase = nb2;
            if (nl < s.nlev) load(nl, p2, nx);
            nb2 = nbase + step;
            seek(nl2, nb2);
            if (nl2 < s.nlev) p2 = point_of(nl2, nb2);
            const int t = cur.t;
            const bool act = cur.act;
            const float dt = cur.dt, lam = cur.lam;
            float bu0 = 0.0f, bu1 = 0.0f;
#pragma unroll
            for (int r = 0; r < RM; r++) {
                bu0 = __fmaf_rn(cur.b0[r], cur.u[r], bu0);
                bu1 = __fmaf_rn(cur.b1[r], cur.u[r], bu1);
            }
            const float al0 = kmb_exp(dt * A0, s.fast), al1 = kmb_exp(dt * A1, s.fast);
            float hn0, hn1;
            if (NDT >= 2) {
                float bacc0 = 0.0f, bacc1 = 0.0f;
                hn0 = 0.0f;
                hn1 = 0.0f;
                int np = 0;
#pragma unroll
                for (int k = 0; k < NDT; k++) {
                    if (!((cur.nb >> k) & 1)) continue;
                    const int q = rix(pb, cur.ppos[k]);
                    const float p0 = ring_h[q], p1 = ring_h[q + 1];
                    const float r0 = pair ? cth * p0 - sth * p1 : p0;
                    const float r1 = sth * p0 + cth * p1;
                    hn0 = __fmaf_rn(al0, r0, hn0);
                    hn1 = __fmaf_rn(al1, r1, hn1);
                    bacc0 += ring_b[q];
                    bacc1 += ring_b[q + 1];
                    np++;
                }
                if (np > 0) {
                    const float bs = (1.0f - lam) * dt / (float)np;
                    hn0 = __fmaf_rn(bs * al0, bacc0, hn0);
                    hn1 = __fmaf_rn(bs * al1, bacc1, hn1);
                }
                const float gm = lam * dt;
                hn0 = __fmaf_rn(gm, bu0, hn0);
                hn1 = __fmaf_rn(gm, bu1, hn1);
            } else {
                // 1D recurrence (reference src/mamba_block.c:384-393)
                float p0 = 0.0f, p1 = 0.0f, pb0 = 0.0f, pb1 = 0.0f;
                if (cur.nb & 1) {
                    const int q = rix(pb, cur.ppos[0]);
                    p0 = ring_h[q]; p1 = ring_h[q + 1];
                    pb0 = ring_b[q]; pb1 = ring_b[q + 1];
                }
                const float r0 = pair ? cth * p0 - sth * p1 : p0;
                const float r1 = sth * p0 + cth * p1;
                const float beta0 = (1.0f - lam) * dt * al0, beta1 = (1.0f - lam) * dt * al1;
                const float gm = lam * dt;
                hn0 = __fmaf_rn(gm, bu0, __fmaf_rn(beta0, pb0, al0 * r0));
                hn1 = __fmaf_rn(gm, bu1, __fmaf_rn(beta1, pb1, al1 * r1));
            }
            // states of absent states (odd N, padding pairs) stay 0 in the ring
            if (!h0ok) { hn0 = 0.0f; bu0 = 0.0f; }
            if (!h1ok) { hn1 = 0.0f; bu1 = 0.0f; }
            if (act) {
                const int q = rix(cb, cur.pos);
                ring_h[q] = hn0; ring_h[q + 1] = hn1;
                ring_b[q] = bu0; ring_b[q + 1] = bu1;
                const int o = t * N;
                if (h0ok) { h[o + n0] = hn0; Bu[o + n0] = bu0; }
                if (h1ok) { h[o + n1] = hn1; Bu[o + n1] = bu1; }
            }
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r >= R) break;
                float part = 0.0f;
                if (h0ok) part = cur.c0[r] * hn0;
                if (h1ok) part = __fmaf_rn(cur.c1[r], hn1, part);
                part = group_sum<GP>(part);
                if (act && ln.pl == 0) y[t * R + r] = part;
            }
        }
        __syncthreads();
    }
}

// Forward for 2D grids with an inner extent W <= 64, N <= 64, R in {1, 2, 4}: a
// systolic column-strip pipeline instead of level barriers.  CTA = item; warp w
// owns columns 8w .. 8w+7 of every row; lane p owns the state pair (2p, 2p+1).
// For each of its columns a lane keeps the previous row's rotated state R(theta)h
// and its B*u product in registers; the left neighbour of its first column comes
// from warp w-1 through shared-memory slots guarded by mbarriers (bounded waits),
// so warps run one row apart and predecessor states never touch memory.  Per point
// the arithmetic is the same as blockscan_fwd_ring's (outer predecessor, then
// inner); y is a transposed butterfly over the 32 pairs.  STAGED: each warp keeps
// its next NSS rows of B, C, u, dt, lambda in flight in shared memory with bulk
// copies (W % 8 == 0, N % 8 == 0: every piece is a whole run of 16-byte units);
// otherwise a row's inputs are loaded at the start of the row.
constexpr int BSS_WC = 8, BSS_K = 4, BSS_NSS = 3;

// Bulk (non-tensor, no multicast) copy global -> this CTA's shared memory, completion on an mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, unsigned bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// Byte layout of one staged row of a strip: B [8][R][N] | C [8][R][N] | u [8][R] | dt [8] | lambda [8],
// each piece rounded up to 16 bytes.
template <typename T>
struct BSStage {
    int offC, offU, offD, offL, bytes;
    __host__ __device__ BSStage(int R, int N, bool has_lam) {
        const int bc = BSS_WC * R * N * (int)sizeof(T);
        auto up = [](int v) { return (v + 15) & ~15; };
        offC = up(bc);
        offU = offC + up(bc);
        offD = offU + up(BSS_WC * R * (int)sizeof(T));
        offL = offD + up(BSS_WC * (int)sizeof(T));
        bytes = offL + (has_lam ? up(BSS_WC * (int)sizeof(T)) : 0);
    }
};

template <typename T, int RP, bool STAGED>
__global__ void __launch_bounds__(256, 1) blockscan_fwd_strips(BSDesc s, int* status) {
    extern __shared__ __align__(16) unsigned char bss_smem[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, S = blockDim.x >> 5;
    const int b = blockIdx.x;
    const int H = s.dims[0], W = s.dims[1];
    const int N = s.N, R = s.R, NR = N * R;
    const int n0 = 2 * lane, n1 = 2 * lane + 1;
    const bool h0ok = n0 < N, h1ok = n1 < N, pair = h1ok;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        kmb_cos_sin(s.theta[lane], &cth, &sth);
    }
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR;
    float* h = s.h + b * L * N;
    float* Bu = s.Bu + b * L * N;
    float* y = s.y + b * L * R;
    // handoff slots [S][K][4][32] (rotated h pair, B*u pair), their barriers, stage barriers, stages
    float* hand = (float*)bss_smem;
    uint64_t* hfull = (uint64_t*)(hand + (size_t)S * BSS_K * 4 * 32);
    uint64_t* hempty = hfull + S * BSS_K;
    uint64_t* sfull = hempty + S * BSS_K;                            // [S][NSS]
    const BSStage<T> sl(R, N, lamp != nullptr);
    // [S][NSS][sl.bytes], 128-byte aligned (bulk copies need 16-byte aligned destinations)
    unsigned char* stages = (unsigned char*)(((uintptr_t)(sfull + S * BSS_NSS) + 127) & ~(uintptr_t)127);
    if (threadIdx.x == 0) {
        for (int i = 0; i < S * BSS_K; i++) {
            mbar_init(smem_u32(&hfull[i]), 1);
            mbar_init(smem_u32(&hempty[i]), 1);
        }
        for (int i = 0; i < S * BSS_NSS; i++) mbar_init(smem_u32(&sfull[i]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int q0 = w * BSS_WC;
    const int ncol = min(BSS_WC, W - q0);
    auto issue = [&](int orow) {
        const int slot = orow % BSS_NSS;
        unsigned char* st = stages + ((size_t)w * BSS_NSS + slot) * sl.bytes;
        const uint32_t fb = smem_u32(&sfull[w * BSS_NSS + slot]);
        const int t0 = orow * W + q0;
        const unsigned bcb = BSS_WC * R * N * sizeof(T), ub = BSS_WC * R * sizeof(T), db = BSS_WC * sizeof(T);
        mbar_expect_tx(fb, 2 * bcb + ub + db + (lamp ? db : 0));
        bulk_load(smem_u32(st), Bp + (size_t)t0 * NR, bcb, fb);
        bulk_load(smem_u32(st + sl.offC), Cp + (size_t)t0 * NR, bcb, fb);
        bulk_load(smem_u32(st + sl.offU), u + (size_t)t0 * R, ub, fb);
        bulk_load(smem_u32(st + sl.offD), dtp + t0, db, fb);
        if (lamp) bulk_load(smem_u32(st + sl.offL), lamp + t0, db, fb);
    };
    int issued = 0;
    if (STAGED && lane == 0)
        for (; issued < BSS_NSS && issued < H; issued++) issue(issued);
    // leaving early: copies in flight must land first (bounded)
    auto drain = [&]() {
        if constexpr (STAGED) {
            if (lane != 0) return;
            for (int j = (issued > BSS_NSS ? issued - BSS_NSS : 0); j < issued; j++)
                mbar_wait(smem_u32(&sfull[w * BSS_NSS + j % BSS_NSS]), (uint32_t)((j / BSS_NSS) & 1));
        }
    };
    // y: lane gl holds value butterfly_index = (column j, rank r) after the reduction
    constexpr int NV = BSS_WC * RP, LPV = 32 / NV;
    const int yidx = butterfly_index<NV, 32>(lane);
    const int yj = yidx / RP, yr = yidx % RP;
    const bool y_lane = (LPV <= 1 || (lane % LPV) == 0) && yj < ncol && yr < R;
    float rh0[BSS_WC], rh1[BSS_WC], rb0[BSS_WC], rb1[BSS_WC];
#pragma unroll
    for (int j = 0; j < BSS_WC; j++) rh0[j] = rh1[j] = rb0[j] = rb1[j] = 0.0f;
    for (int o = 0; o < H; o++) {
        // ---- inputs of the row
        float uu[BSS_WC][RP], bb0[BSS_WC][RP], bb1[BSS_WC][RP], cc0[BSS_WC][RP], cc1[BSS_WC][RP];
        float dtv[BSS_WC], lmv[BSS_WC];
        if constexpr (STAGED) {
            const int slot = o % BSS_NSS;
            if (!mbar_wait(smem_u32(&sfull[w * BSS_NSS + slot]), (uint32_t)((o / BSS_NSS) & 1))) {
                set_status(status, KMB_ERR_TIMEOUT_FULL);
                drain();
                return;
            }
            const unsigned char* st = stages + ((size_t)w * BSS_NSS + slot) * sl.bytes;
            const T* sB = (const T*)st;
            const T* sC = (const T*)(st + sl.offC);
            const T* sU = (const T*)(st + sl.offU);
            const T* sD = (const T*)(st + sl.offD);
            const T* sL = (const T*)(st + sl.offL);
#pragma unroll
            for (int j = 0; j < BSS_WC; j++) {
                dtv[j] = ldv(sD + j);
                lmv[j] = lamp ? ldv(sL + j) : s.deflam;
#pragma unroll
                for (int r = 0; r < RP; r++) {
                    const bool rr = r < R;
                    const int c = j * NR + (rr ? r : 0) * N;
                    uu[j][r] = rr ? ldv(sU + j * R + r) : 0.0f;
                    bb0[j][r] = rr && h0ok ? ldv(sB + c + n0) : 0.0f;
                    bb1[j][r] = rr && h1ok ? ldv(sB + c + n1) : 0.0f;
                    cc0[j][r] = rr && h0ok ? ldv(sC + c + n0) : 0.0f;
                    cc1[j][r] = rr && h1ok ? ldv(sC + c + n1) : 0.0f;
                }
            }
            // the stage is read: refill it with row o + NSS
            __syncwarp();
            if (lane == 0 && o + BSS_NSS < H) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(o + BSS_NSS);
                issued = o + BSS_NSS + 1;
            }
        } else {
#pragma unroll
            for (int j = 0; j < BSS_WC; j++) {
                const int t = o * W + q0 + (j < ncol ? j : 0);
                dtv[j] = ldv(dtp + t);
                lmv[j] = lamp ? ldv(lamp + t) : s.deflam;
#pragma unroll
                for (int r = 0; r < RP; r++) {
                    const bool rr = r < R;
                    const int c = t * NR + (rr ? r : 0) * N;
                    uu[j][r] = rr ? ldv(u + t * R + r) : 0.0f;
                    bb0[j][r] = rr && h0ok ? ldv(Bp + c + n0) : 0.0f;
                    bb1[j][r] = rr && h1ok ? ldv(Bp + c + n1) : 0.0f;
                    cc0[j][r] = rr && h0ok ? ldv(Cp + c + n0) : 0.0f;
                    cc1[j][r] = rr && h1ok ? ldv(Cp + c + n1) : 0.0f;
                }
            }
        }
        // ---- left neighbour of the first column, from warp w-1
        const int hs = o & (BSS_K - 1);
        const uint32_t hph = (uint32_t)((o / BSS_K) & 1);
        float lh0 = 0.0f, lh1 = 0.0f, lb0 = 0.0f, lb1 = 0.0f;
        if (w > 0) {
            if (!mbar_wait(smem_u32(&hfull[w * BSS_K + hs]), hph)) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                drain();
                return;
            }
            const float* src = hand + ((size_t)w * BSS_K + hs) * 128;
            lh0 = src[lane];
            lh1 = src[32 + lane];
            lb0 = src[64 + lane];
            lb1 = src[96 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hempty[w * BSS_K + hs]));
        }
        float prod[BSS_WC][RP];
#pragma unroll
        for (int j = 0; j < BSS_WC; j++) {
#pragma unroll
            for (int r = 0; r < RP; r++) prod[j][r] = 0.0f;
            if (j >= ncol) continue;
            const int t = o * W + q0 + j;
            const float dt = dtv[j], lam = lmv[j];
            float bu0 = 0.0f, bu1 = 0.0f;
#pragma unroll
            for (int r = 0; r < RP; r++) {
                bu0 = __fmaf_rn(bb0[j][r], uu[j][r], bu0);
                bu1 = __fmaf_rn(bb1[j][r], uu[j][r], bu1);
            }
            const float al0 = kmb_exp(dt * A0, s.fast), al1 = kmb_exp(dt * A1, s.fast);
            float hn0 = 0.0f, hn1 = 0.0f, bacc0 = 0.0f, bacc1 = 0.0f;
            int np = 0;
            if (o > 0) {   // outer predecessor (o-1, q): this column's ring entry (previous row)
                hn0 = __fmaf_rn(al0, rh0[j], hn0);
                hn1 = __fmaf_rn(al1, rh1[j], hn1);
                bacc0 += rb0[j];
                bacc1 += rb1[j];
                np++;
            }
            if (q0 + j > 0) {   // inner predecessor (o, q-1): the previous column (this row)
                const float p0 = j == 0 ? lh0 : rh0[j == 0 ? 0 : j - 1];
                const float p1 = j == 0 ? lh1 : rh1[j == 0 ? 0 : j - 1];
                const float q0b = j == 0 ? lb0 : rb0[j == 0 ? 0 : j - 1];
                const float q1b = j == 0 ? lb1 : rb1[j == 0 ? 0 : j - 1];
                hn0 = __fmaf_rn(al0, p0, hn0);
                hn1 = __fmaf_rn(al1, p1, hn1);
                bacc0 += q0b;
                bacc1 += q1b;
                np++;
            }
            if (np > 0) {
                const float bs = (1.0f - lam) * dt / (float)np;
                hn0 = __fmaf_rn(bs * al0, bacc0, hn0);
                hn1 = __fmaf_rn(bs * al1, bacc1, hn1);
            }
            const float gm = lam * dt;
            hn0 = __fmaf_rn(gm, bu0, hn0);
            hn1 = __fmaf_rn(gm, bu1, hn1);
            if (!h0ok) { hn0 = 0.0f; bu0 = 0.0f; }
            if (!h1ok) { hn1 = 0.0f; bu1 = 0.0f; }
            const int ot = t * N;
            if (h0ok) { h[ot + n0] = hn0; Bu[ot + n0] = bu0; }
            if (h1ok) { h[ot + n1] = hn1; Bu[ot + n1] = bu1; }
            // the predecessor form read by the next row / column: R(theta) h and B*u
            rh0[j] = pair ? cth * hn0 - sth * hn1 : hn0;
            rh1[j] = sth * hn0 + cth * hn1;
            rb0[j] = bu0;
            rb1[j] = bu1;
#pragma unroll
            for (int r = 0; r < RP; r++) {
                float part = 0.0f;
                if (h0ok) part = cc0[j][r] * hn0;
                if (h1ok) part = __fmaf_rn(cc1[j][r], hn1, part);
                prod[j][r] = part;
            }
        }
        // ---- right boundary to warp w+1
        if (w + 1 < S) {
            if (o >= BSS_K && !mbar_wait(smem_u32(&hempty[(w + 1) * BSS_K + hs]), hph ^ 1)) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                drain();
                return;
            }
            float* dst = hand + ((size_t)(w + 1) * BSS_K + hs) * 128;
            const int lj = ncol - 1;
            float a0 = 0.0f, a1 = 0.0f, c0 = 0.0f, c1 = 0.0f;
#pragma unroll
            for (int j = 0; j < BSS_WC; j++)
                if (j == lj) { a0 = rh0[j]; a1 = rh1[j]; c0 = rb0[j]; c1 = rb1[j]; }
            dst[lane] = a0;
            dst[32 + lane] = a1;
            dst[64 + lane] = c0;
            dst[96 + lane] = c1;
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hfull[(w + 1) * BSS_K + hs]));
        }
        // ---- y[t, r] = sum over the states
        {
            float v[NV];
#pragma unroll
            for (int j = 0; j < BSS_WC; j++)
#pragma unroll
                for (int r = 0; r < RP; r++) v[j * RP + r] = prod[j][r];
            const float sum = butterfly<NV, 32>(v, lane);
            if (y_lane) y[(o * W + q0 + yj) * R + yr] = sum;
        }
    }
}

struct BSGrad {
    const float* dy;
    float *dB, *dC, *du, *ddt, *dlam;
    float* G;     // scratch [batch, L, N]
    float* pA;    // scratch [batch, N]
    float* pth;   // scratch [batch, 32]
    // NG > 1: per-group partials [NG][batch][L][R] and [NG][batch][L] (x2)
    float *pdu, *pddt, *pdlam;
    int overwrite;   // 1: dB, dC, du, ddt, dlambda are assigned, not accumulated (strip backward only)
};

template <typename T, int GP>
__global__ void __launch_bounds__(512) blockscan_bwd_generic(BSDesc s, BSGrad g) {
    using Ln = BSLanes<GP>;
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0, n1 = ln.n1;
    const bool h0ok = ln.h0ok, h1ok = ln.h1ok, pair = ln.pair;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R, nd = s.nd < 1 ? 1 : s.nd;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    const long long L = s.L;
    const T* u = (const T*)s.u + b * L * R;
    const T* dtp = (const T*)s.dt + b * L;
    const T* lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* Bp = (const T*)s.B + b * L * NR;
    const T* Cp = (const T*)s.C + b * L * NR;
    const float* h = s.h + b * L * N;
    const float* Bu = s.Bu + b * L * N;
    const float* dy = g.dy + b * L * R;
    float* G = g.G + b * L * N;
    float* dBi = g.dB + b * L * NR;
    float* dCi = g.dC + b * L * NR;
    // du / ddt / dlambda: accumulate in place (one group), or this group's partials
    const bool direct = s.NG == 1;
    const long long gofs = (long long)ln.g * s.batch;
    float* du = direct ? g.du + b * L * R : g.pdu + (gofs + b) * L * R;
    float* ddt = direct ? (g.ddt ? g.ddt + b * L : nullptr) : g.pddt + (gofs + b) * L;
    float* dlam = direct ? (g.dlam ? g.dlam + b * L : nullptr) : g.pdlam + (gofs + b) * L;
    float gA0 = 0.0f, gA1 = 0.0f, gth = 0.0f;
    int dims[BS_MAXND], strides[BS_MAXND];
    if (s.nd >= 1) {
        for (int k = 0; k < nd; k++) { dims[k] = s.dims[k]; strides[k] = s.strides[k]; }
    } else {
        dims[0] = (int)L;
        strides[0] = 1;
    }
    for (int lev = s.nlev - 1; lev >= 0; lev--) {
        const int beg = s.lev_start[lev], end = s.lev_start[lev + 1];
        for (int base = beg + warp * Ln::PPW; base < end; base += nw * Ln::PPW) {
            const bool act = base + ln.ps < end;
            const int t = s.lev_pts[act ? base + ln.ps : base];
            // inactive point slots compute on a duplicate point and store nothing
            const bool x0 = act && h0ok, x1 = act && h1ok;
            int idx[BS_MAXND];
            int npt = 0;
            for (int k = 0; k < nd; k++) {
                idx[k] = (t / strides[k]) % dims[k];
                npt += idx[k] > 0;
            }
            const float dt = ldv(dtp + t);
            const float lam = lamp ? ldv(lamp + t) : s.deflam;
            // pull from successors s = t + e_k
            float a0 = 0.0f, a1 = 0.0f, ab0 = 0.0f, ab1 = 0.0f;
            for (int k = 0; k < nd; k++) {
                if (idx[k] >= dims[k] - 1) continue;
                const int sp = t + strides[k];
                const float dts = ldv(dtp + sp);
                const float lams = lamp ? ldv(lamp + sp) : s.deflam;
                const int nps = npt + (idx[k] == 0 ? 1 : 0);
                const float al0 = kmb_exp(dts * A0, s.fast), al1 = kmb_exp(dts * A1, s.fast);
                const float coef = (1.0f - lams) * dts / (float)nps;
                const float G0 = h0ok ? G[sp * N + n0] : 0.0f;
                const float G1 = h1ok ? G[sp * N + n1] : 0.0f;
                a0 += al0 * G0;
                a1 += al1 * G1;
                ab0 += coef * al0 * G0;
                ab1 += coef * al1 * G1;
            }
            float gh0 = pair ? cth * a0 + sth * a1 : a0;
            float gh1 = -sth * a0 + cth * a1;
            const int o = t * N;
            const float ht0 = h0ok ? h[o + n0] : 0.0f, ht1 = h1ok ? h[o + n1] : 0.0f;
            if (pair && act) {
                const float hat0 = cth * ht0 - sth * ht1, hat1 = sth * ht0 + cth * ht1;
                gth += -a0 * hat1 + a1 * hat0;
            }
            for (int r = 0; r < R; r++) {
                const float dyr = dy[t * R + r];
                const int c0 = t * NR + r * N;
                if (h0ok) {
                    gh0 += ldv(Cp + c0 + n0) * dyr;
                    if (act) dCi[c0 + n0] += dyr * ht0;
                }
                if (h1ok) {
                    gh1 += ldv(Cp + c0 + n1) * dyr;
                    if (act) dCi[c0 + n1] += dyr * ht1;
                }
            }
            if (x0) G[o + n0] = gh0;
            if (x1) G[o + n1] = gh1;
            const float bu0 = h0ok ? Bu[o + n0] : 0.0f, bu1 = h1ok ? Bu[o + n1] : 0.0f;
            const float gam = lam * dt;
            const float gbu0 = gam * gh0 + ab0, gbu1 = gam * gh1 + ab1;
            for (int r = 0; r < R; r++) {
                const float ur = ldv(u + t * R + r);
                const int c0 = t * NR + r * N;
                float part = 0.0f;
                if (h0ok) {
                    if (act) dBi[c0 + n0] += gbu0 * ur;
                    part += gbu0 * ldv(Bp + c0 + n0);
                }
                if (h1ok) {
                    if (act) dBi[c0 + n1] += gbu1 * ur;
                    part += gbu1 * ldv(Bp + c0 + n1);
                }
                part = group_sum<GP>(part);
                if (act && ln.pl == 0) {
                    if (direct) du[t * R + r] += part;
                    else du[t * R + r] = part;
                }
            }
            float gdt = lam * (bu0 * gh0 + bu1 * gh1);
            float glam = dt * (bu0 * gh0 + bu1 * gh1);
            if (npt > 0) {
                float sh0 = 0.0f, sh1 = 0.0f, sb0 = 0.0f, sb1 = 0.0f;
                for (int k = 0; k < nd; k++) {
                    if (idx[k] == 0) continue;
                    const long long q = (long long)(t - strides[k]) * N;
                    const float p0 = h0ok ? h[q + n0] : 0.0f, p1 = h1ok ? h[q + n1] : 0.0f;
                    sh0 += pair ? cth * p0 - sth * p1 : p0;
                    sh1 += sth * p0 + cth * p1;
                    if (h0ok) sb0 += Bu[q + n0];
                    if (h1ok) sb1 += Bu[q + n1];
                }
                const float inv = 1.0f / (float)npt;
                const float sc = (1.0f - lam) * dt * inv;
                const float z0 = dt * A0, z1 = dt * A1;
                const float al0 = kmb_exp(z0, s.fast), al1 = kmb_exp(z1, s.fast);
                const float dal0 = (sh0 + sc * sb0) * gh0, dal1 = (sh1 + sc * sb1) * gh1;
                const float dz0 = h0ok ? kmb_dexp(z0, al0, s.fast) * dal0 : 0.0f;
                const float dz1 = h1ok ? kmb_dexp(z1, al1, s.fast) * dal1 : 0.0f;
                gdt += dz0 * A0 + dz1 * A1;
                if (act) {
                    gA0 += dz0 * dt;
                    gA1 += dz1 * dt;
                }
                const float ds = al0 * sb0 * gh0 + al1 * sb1 * gh1;
                gdt += (1.0f - lam) * inv * ds;
                glam -= dt * inv * ds;
            }
            gdt = group_sum<GP>(gdt);
            glam = group_sum<GP>(glam);
            if (act && ln.pl == 0) {
                if (direct) {
                    if (ddt) ddt[t] += gdt;
                    if (dlam) dlam[t] += glam;
                } else {
                    ddt[t] = gdt;
                    dlam[t] = glam;
                }
            }
        }
        __syncthreads();
    }
    // per-(item, group) partials of dA and dtheta: sum the warps' and point
    // slots' accumulators in a fixed order
    __shared__ float sA[16 * 32][2];
    __shared__ float sT[16 * 32];
    const int tid = threadIdx.x;
    sA[tid][0] = gA0;
    sA[tid][1] = gA1;
    sT[tid] = gth;
    __syncthreads();
    if (tid < GP) {
        float t0 = 0.0f, t1 = 0.0f, tt = 0.0f;
        for (int j = 0; j < nw * Ln::PPW; j++) {
            const int src = (j / Ln::PPW) * 32 + (j % Ln::PPW) * GP + tid;  // (warp, point slot, pair tid)
            t0 += sA[src][0];
            t1 += sA[src][1];
            tt += sT[src];
        }
        const int p = ln.g * GP + tid;
        if (2 * p < N) g.pA[(long long)b * N + 2 * p] = t0;
        if (2 * p + 1 < N) g.pA[(long long)b * N + 2 * p + 1] = t1;
        if (p < 32) g.pth[(long long)b * 32 + p] = tt;
    }
}

// Backward for grids of NDT <= 3 dimensions and rank R <= RM <= 4: every load
// of a point (successors' adjoints and steps, predecessors' states, its own
// inputs and the old gradient values it accumulates into) is issued before
// any store, so a point costs one memory round trip instead of several.
template <typename T, int GP, int RM, int NDT>
__global__ void __launch_bounds__(512) blockscan_bwd_kernel(BSDesc s, BSGrad g) {
    using Ln = BSLanes<GP>;
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0, n1 = ln.n1;
    const bool h0ok = ln.h0ok, h1ok = ln.h1ok, pair = ln.pair;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR;
    const float* __restrict__ h = s.h + b * L * N;
    const float* __restrict__ Bu = s.Bu + b * L * N;
    const float* __restrict__ dy = g.dy + b * L * R;
    float* G = g.G + b * L * N;
    float* dB = g.dB + b * L * NR;
    float* dC = g.dC + b * L * NR;
    const bool direct = s.NG == 1;
    const long long gofs = (long long)ln.g * s.batch;
    float* du = direct ? g.du + b * L * R : g.pdu + (gofs + b) * L * R;
    float* ddt = direct ? (g.ddt ? g.ddt + b * L : nullptr) : g.pddt + (gofs + b) * L;
    float* dlam = direct ? (g.dlam ? g.dlam + b * L : nullptr) : g.pdlam + (gofs + b) * L;
    float gA0 = 0.0f, gA1 = 0.0f, gth = 0.0f;
    int dims[NDT], strides[NDT];
#pragma unroll
    for (int k = 0; k < NDT; k++) {
        dims[k] = NDT == 1 ? (int)L : s.dims[k];
        strides[k] = NDT == 1 ? 1 : s.strides[k];
    }
    for (int lev = s.nlev - 1; lev >= 0; lev--) {
        const int beg = s.lev_start[lev], end = s.lev_start[lev + 1];
        for (int base = beg + warp * Ln::PPW; base < end; base += nw * Ln::PPW) {
            const bool act = base + ln.ps < end;
            const int t = s.lev_pts[act ? base + ln.ps : base];
            const bool x0 = act && h0ok, x1 = act && h1ok;
            // neighbour mask from the plan (bit k: predecessor along k, bit 8 + k: successor)
            const int nbm = s.nbr[t];
            const int npt = __popc(nbm & 0xff);
            // ---- loads
            const float dt = ldv(dtp + t);
            const float lam = lamp ? ldv(lamp + t) : s.deflam;
            bool hs[NDT], hp[NDT];
            float sdt[NDT], slam[NDT], sG0[NDT], sG1[NDT], ph0[NDT], ph1[NDT], pb0[NDT], pb1[NDT];
#pragma unroll
            for (int k = 0; k < NDT; k++) {
                hs[k] = (nbm >> (8 + k)) & 1;
                const int sp = hs[k] ? t + strides[k] : t;
                sdt[k] = ldv(dtp + sp);
                slam[k] = lamp ? ldv(lamp + sp) : s.deflam;
                sG0[k] = h0ok && hs[k] ? G[sp * N + n0] : 0.0f;
                sG1[k] = h1ok && hs[k] ? G[sp * N + n1] : 0.0f;
                hp[k] = (nbm >> k) & 1;
                const int q = (hp[k] ? t - strides[k] : t) * N;
                ph0[k] = h0ok ? h[q + n0] : 0.0f;
                ph1[k] = h1ok ? h[q + n1] : 0.0f;
                pb0[k] = h0ok ? Bu[q + n0] : 0.0f;
                pb1[k] = h1ok ? Bu[q + n1] : 0.0f;
            }
            const int o = t * N;
            const float ht0 = h0ok ? h[o + n0] : 0.0f, ht1 = h1ok ? h[o + n1] : 0.0f;
            const float bu0 = h0ok ? Bu[o + n0] : 0.0f, bu1 = h1ok ? Bu[o + n1] : 0.0f;
            float dyv[RM], uu[RM], c0[RM], c1[RM], b0[RM], b1[RM];
#pragma unroll
            for (int r = 0; r < RM; r++) {
                const bool rr = r < R;
                const int c = t * NR + (rr ? r : 0) * N;
                dyv[r] = rr ? dy[t * R + r] : 0.0f;
                uu[r] = rr ? ldv(u + t * R + r) : 0.0f;
                c0[r] = rr && h0ok ? ldv(Cp + c + n0) : 0.0f;
                c1[r] = rr && h1ok ? ldv(Cp + c + n1) : 0.0f;
                b0[r] = rr && h0ok ? ldv(Bp + c + n0) : 0.0f;
                b1[r] = rr && h1ok ? ldv(Bp + c + n1) : 0.0f;
            }
            // ---- pull from successors s = t + e_k
            float a0 = 0.0f, a1 = 0.0f, ab0 = 0.0f, ab1 = 0.0f;
#pragma unroll
            for (int k = 0; k < NDT; k++) {
                if (!hs[k]) continue;
                const int nps = npt + (((nbm >> k) & 1) ? 0 : 1);
                const float al0 = kmb_exp(sdt[k] * A0, s.fast), al1 = kmb_exp(sdt[k] * A1, s.fast);
                const float coef = (1.0f - slam[k]) * sdt[k] / (float)nps;
                a0 += al0 * sG0[k];
                a1 += al1 * sG1[k];
                ab0 += coef * al0 * sG0[k];
                ab1 += coef * al1 * sG1[k];
            }
            float gh0 = pair ? cth * a0 + sth * a1 : a0;
            float gh1 = -sth * a0 + cth * a1;
            if (pair && act) {
                const float hat0 = cth * ht0 - sth * ht1, hat1 = sth * ht0 + cth * ht1;
                gth += -a0 * hat1 + a1 * hat0;
            }
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r >= R) continue;
                if (h0ok) gh0 += c0[r] * dyv[r];
                if (h1ok) gh1 += c1[r] * dyv[r];
            }
            const float gam = lam * dt;
            const float gbu0 = gam * gh0 + ab0, gbu1 = gam * gh1 + ab1;
            float gdt = lam * (bu0 * gh0 + bu1 * gh1);
            float glam = dt * (bu0 * gh0 + bu1 * gh1);
            if (npt > 0) {
                float sh0 = 0.0f, sh1 = 0.0f, sb0 = 0.0f, sb1 = 0.0f;
#pragma unroll
                for (int k = 0; k < NDT; k++) {
                    if (!hp[k]) continue;
                    sh0 += pair ? cth * ph0[k] - sth * ph1[k] : ph0[k];
                    sh1 += sth * ph0[k] + cth * ph1[k];
                    sb0 += pb0[k];
                    sb1 += pb1[k];
                }
                const float inv = 1.0f / (float)npt;
                const float sc = (1.0f - lam) * dt * inv;
                const float z0 = dt * A0, z1 = dt * A1;
                const float al0 = kmb_exp(z0, s.fast), al1 = kmb_exp(z1, s.fast);
                const float dal0 = (sh0 + sc * sb0) * gh0, dal1 = (sh1 + sc * sb1) * gh1;
                const float dz0 = h0ok ? kmb_dexp(z0, al0, s.fast) * dal0 : 0.0f;
                const float dz1 = h1ok ? kmb_dexp(z1, al1, s.fast) * dal1 : 0.0f;
                gdt += dz0 * A0 + dz1 * A1;
                if (act) {
                    gA0 += dz0 * dt;
                    gA1 += dz1 * dt;
                }
                const float ds = al0 * sb0 * gh0 + al1 * sb1 * gh1;
                gdt += (1.0f - lam) * inv * ds;
                glam -= dt * inv * ds;
            }
            // ---- stores
            if (x0) G[o + n0] = gh0;
            if (x1) G[o + n1] = gh1;
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r >= R) continue;
                const int c = t * NR + r * N;
                if (x0) {
                    // one addition each (old + value): no read of the old value in the chain
                    atomicAdd(&dC[c + n0], dyv[r] * ht0);
                    atomicAdd(&dB[c + n0], gbu0 * uu[r]);
                }
                if (x1) {
                    atomicAdd(&dC[c + n1], dyv[r] * ht1);
                    atomicAdd(&dB[c + n1], gbu1 * uu[r]);
                }
                float part = 0.0f;
                if (h0ok) part += gbu0 * b0[r];
                if (h1ok) part += gbu1 * b1[r];
                part = group_sum<GP>(part);
                if (act && ln.pl == 0) {
                    if (direct) du[t * R + r] += part;
                    else du[t * R + r] = part;
                }
            }
            gdt = group_sum<GP>(gdt);
            glam = group_sum<GP>(glam);
            if (act && ln.pl == 0) {
                if (direct) {
                    if (ddt) ddt[t] += gdt;
                    if (dlam) dlam[t] += glam;
                } else {
                    ddt[t] = gdt;
                    dlam[t] = glam;
                }
            }
        }
        __syncthreads();
    }
    __shared__ float sA[16 * 32][2];
    __shared__ float sT[16 * 32];
    const int tid = threadIdx.x;
    sA[tid][0] = gA0;
    sA[tid][1] = gA1;
    sT[tid] = gth;
    __syncthreads();
    if (tid < GP) {
        float t0 = 0.0f, t1 = 0.0f, tt = 0.0f;
        for (int j = 0; j < nw * Ln::PPW; j++) {
            const int src = (j / Ln::PPW) * 32 + (j % Ln::PPW) * GP + tid;
            t0 += sA[src][0];
            t1 += sA[src][1];
            tt += sT[src];
        }
        const int p = ln.g * GP + tid;
        if (2 * p < N) g.pA[(long long)b * N + 2 * p] = t0;
        if (2 * p + 1 < N) g.pA[(long long)b * N + 2 * p + 1] = t1;
        if (p < 32) g.pth[(long long)b * 32 + p] = tt;
    }
}

// Backward for 2D grids, R in {1, 2, 4}: a systolic reverse column-strip
// pipeline, the mirror of blockscan_fwd_strips, with the state pairs split
// into groups as in the level kernels (CTA = (item, group of GP pairs)).
// Strips of CW columns are numbered from the right; a warp carries SPW = 32 /
// GP strips at once (lane = (slot, pair)), slot ss working one row behind slot
// ss - 1, rows bottom to top and columns right to left.  What a point hands to
// its predecessors -- alpha * g_h and coef * alpha * g_h per state, the exact
// terms the level kernel pulls from a successor -- stays in registers for the
// outer axis (same column, next row), moves along the strip in registers, to
// the next slot by a shuffle, and to the next warp through mbarrier-guarded
// shared-memory slots (bounded waits).  So the state adjoints never touch
// memory; h and B*u of a point and its predecessors are read back from the
// forward, and the next row's loads are issued before the current row's
// arithmetic.  Per point the arithmetic is the level kernel's.
constexpr int BSB_K = 4;

__device__ __forceinline__ float2 ld2(const float* p) { return *(const float2*)p; }
__device__ __forceinline__ float2 ld2(const __nv_bfloat16* p) {
    return __bfloat1622float2(*(const __nv_bfloat162*)p);
}

// One column's loads for a row: own h and B*u, the outer predecessor's, the inner
// predecessor's (last column of the strip only; the others take the next
// column's own values), and the point's inputs.  Pairs are one vector load each.
template <int RP>
struct BSBCol {
    float dt, lam;
    float2 ht, bu, uh, ub, lh, lb;
    float dy[RP], u[RP];
    float2 b[RP], c[RP];
};

template <typename T, int GP, int RP, int CW, bool OVW, bool FULL>
__global__ void __launch_bounds__(256, 1) blockscan_bwd_strips(BSDesc s, BSGrad g, int* status) {
    extern __shared__ __align__(16) unsigned char bsb_smem[];
    constexpr int SPW = 32 / GP;
    using Ln = BSLanes<GP>;
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0;
    // N is even: a pair is whole or absent; FULL (N a multiple of 2 GP): every lane has one
    const bool hok = FULL || ln.h0ok;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int ss = ln.ps, pl = ln.pl;
    const int H = s.dims[0], W = s.dims[1];
    constexpr int R = RP;   // the rank is a template parameter here
    const int N = s.N, NR = N * R;
    const int nstrips = (W + CW - 1) / CW;
    const int st = w * SPW + ss;
    const int qb = W - 1 - st * CW;   // rightmost column of the strip
    const float A0 = hok ? s.A[n0] : 0.0f, A1 = hok ? s.A[n0 + 1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (hok) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR + n0;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR + n0;
    const float* __restrict__ h = s.h + b * L * N + n0;
    const float* __restrict__ Bu = s.Bu + b * L * N + n0;
    const float* __restrict__ dy = g.dy + b * L * R;
    float* dB = g.dB + b * L * NR + n0;
    float* dC = g.dC + b * L * NR + n0;
    const bool direct = s.NG == 1;
    const long long gofs = (long long)ln.g * s.batch;
    float* du = direct ? g.du + b * L * R : g.pdu + (gofs + b) * L * R;
    float* ddt = direct ? (g.ddt ? g.ddt + b * L : nullptr) : g.pddt + (gofs + b) * L;
    float* dlam = direct ? (g.dlam ? g.dlam + b * L : nullptr) : g.pdlam + (gofs + b) * L;
    const bool assign = !direct || OVW;

    // handoff slots [nw][K][4][GP] (P pair, Q pair of a strip's leftmost column), then their barriers
    float* hand = (float*)bsb_smem;
    uint64_t* hfull = (uint64_t*)(hand + (size_t)nw * BSB_K * 4 * GP);
    uint64_t* hempty = hfull + nw * BSB_K;
    float* red = (float*)(hempty + nw * BSB_K);   // [nw * 32][3]: dA pair and dtheta partials
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw * BSB_K; i++) {
            mbar_init(smem_u32(&hfull[i]), 1);
            mbar_init(smem_u32(&hempty[i]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const float2 z2 = make_float2(0.0f, 0.0f);
    // Rows and columns outside the grid (pipeline fill and drain, a partial last strip) are clamped
    // into it: their loads are valid and their results are never stored.  An absent predecessor
    // loads as zeros, so the sums over predecessors need no branch.
    auto load_row = [&](BSBCol<RP>* c, int rr) {
        const int o = min(max(H - 1 - rr, 0), H - 1);
#pragma unroll
        for (int j = 0; j < CW; j++) {
            const int q = max(qb - j, 0);
            const int t = o * W + q;
            BSBCol<RP>& x = c[j];
            x.dt = ldv(dtp + t);
            x.lam = lamp ? ldv(lamp + t) : s.deflam;
            const float* hp = h + t * N;
            const float* bp = Bu + t * N;
            x.ht = hok ? ld2(hp) : z2;
            x.bu = hok ? ld2(bp) : z2;
            x.uh = hok && o > 0 ? ld2(hp - W * N) : z2;
            x.ub = hok && o > 0 ? ld2(bp - W * N) : z2;
            if (j == CW - 1) {
                x.lh = hok && q > 0 ? ld2(hp - N) : z2;
                x.lb = hok && q > 0 ? ld2(bp - N) : z2;
            }
            if constexpr (RP == 1) {
                x.dy[0] = dy[t];
                x.u[0] = ldv(u + t);
            } else {
#pragma unroll
                for (int r = 0; r < RP; r += 2) {
                    const float2 d2 = ld2(dy + t * R + r), u2 = ld2(u + t * R + r);
                    x.dy[r] = d2.x;
                    x.dy[r + 1] = d2.y;
                    x.u[r] = u2.x;
                    x.u[r + 1] = u2.y;
                }
            }
#pragma unroll
            for (int r = 0; r < RP; r++) {
                x.b[r] = hok ? ld2(Bp + t * NR + r * N) : z2;
                x.c[r] = hok ? ld2(Cp + t * NR + r * N) : z2;
            }
        }
    };

    float PO0[CW], PO1[CW], QO0[CW], QO1[CW];   // from the outer successor (same column, row below)
#pragma unroll
    for (int j = 0; j < CW; j++) PO0[j] = PO1[j] = QO0[j] = QO1[j] = 0.0f;
    float ob0 = 0.0f, ob1 = 0.0f, oq0 = 0.0f, oq1 = 0.0f;   // this slot's output to the strip on its left
    float gA0 = 0.0f, gA1 = 0.0f, gth = 0.0f;
    // two row buffers used in turn (no register copy that would wait for the prefetch to land)
    BSBCol<RP> bufA[CW], bufB[CW];
    load_row(bufA, -ss);
    const int nsteps = H + SPW - 1;
    auto step = [&](const int i, BSBCol<RP>* cur, BSBCol<RP>* nxt) -> bool {
        const int rr = i - ss;
        const bool act = st < nstrips && rr >= 0 && rr < H;
        const int o = H - 1 - rr;
        load_row(nxt, rr + 1);
        // ---- inner successor of the rightmost column: the strip on the right, same row
        float ip0 = __shfl_up_sync(0xffffffffu, ob0, GP);
        float ip1 = __shfl_up_sync(0xffffffffu, ob1, GP);
        float iq0 = __shfl_up_sync(0xffffffffu, oq0, GP);
        float iq1 = __shfl_up_sync(0xffffffffu, oq1, GP);
        if (ss == 0) ip0 = ip1 = iq0 = iq1 = 0.0f;
        if (w > 0 && i < H) {   // warp-uniform: slot 0 takes row i of warp w - 1's last strip
            const int hs = i & (BSB_K - 1);
            if (!mbar_wait(smem_u32(&hfull[w * BSB_K + hs]), (uint32_t)((i / BSB_K) & 1))) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                return false;
            }
            if (ss == 0) {
                const float* src = hand + ((size_t)w * BSB_K + hs) * 4 * GP;
                ip0 = src[pl];
                ip1 = src[GP + pl];
                iq0 = src[2 * GP + pl];
                iq1 = src[3 * GP + pl];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hempty[w * BSB_K + hs]));
        }
#pragma unroll
        for (int j = 0; j < CW; j++) {
            const int q = qb - j;
            const bool pa = act && q >= 0;
            const BSBCol<RP>& x = cur[j];
            const int t = pa ? o * W + q : 0;
            const bool up = o > 0, lf = q > 0;
            const int npt = (int)up + (int)lf;
            const float ht0 = x.ht.x, ht1 = x.ht.y;
            // ---- successors: outer (row below) first, then inner (column to the right)
            const float a0 = PO0[j] + ip0, a1 = PO1[j] + ip1;
            const float ab0 = QO0[j] + iq0, ab1 = QO1[j] + iq1;
            float gh0 = cth * a0 + sth * a1;
            float gh1 = -sth * a0 + cth * a1;
            if (pa) {
                const float hat0 = cth * ht0 - sth * ht1, hat1 = sth * ht0 + cth * ht1;
                gth += -a0 * hat1 + a1 * hat0;
            }
#pragma unroll
            for (int r = 0; r < RP; r++) {
                gh0 += x.c[r].x * x.dy[r];
                gh1 += x.c[r].y * x.dy[r];
            }
            const float dt = x.dt, lam = x.lam;
            const float bu0 = x.bu.x, bu1 = x.bu.y;
            const float gam = lam * dt;
            const float gbu0 = gam * gh0 + ab0, gbu1 = gam * gh1 + ab1;
            float gdt = lam * (bu0 * gh0 + bu1 * gh1);
            float glam = dt * (bu0 * gh0 + bu1 * gh1);
            // predecessors (absent ones are zeros; with none, every term below is zero)
            const float2 lh = !lf ? z2 : j + 1 < CW ? cur[j + 1 < CW ? j + 1 : j].ht : x.lh;
            const float2 lb = !lf ? z2 : j + 1 < CW ? cur[j + 1 < CW ? j + 1 : j].bu : x.lb;
            float sh0 = 0.0f, sh1 = 0.0f, sb0 = 0.0f, sb1 = 0.0f;
            sh0 += cth * x.uh.x - sth * x.uh.y;
            sh1 += sth * x.uh.x + cth * x.uh.y;
            sb0 += x.ub.x;
            sb1 += x.ub.y;
            sh0 += cth * lh.x - sth * lh.y;
            sh1 += sth * lh.x + cth * lh.y;
            sb0 += lb.x;
            sb1 += lb.y;
            const float fnp = (float)max(npt, 1);
            const float inv = 1.0f / fnp;
            const float sc = (1.0f - lam) * dt * inv;
            const float z0 = dt * A0, z1 = dt * A1;
            const float al0 = kmb_exp(z0, s.fast), al1 = kmb_exp(z1, s.fast);
            const float dal0 = (sh0 + sc * sb0) * gh0, dal1 = (sh1 + sc * sb1) * gh1;
            const float dz0 = hok ? kmb_dexp(z0, al0, s.fast) * dal0 : 0.0f;
            const float dz1 = hok ? kmb_dexp(z1, al1, s.fast) * dal1 : 0.0f;
            gdt += dz0 * A0 + dz1 * A1;
            if (pa) {
                gA0 += dz0 * dt;
                gA1 += dz1 * dt;
            }
            const float ds = al0 * sb0 * gh0 + al1 * sb1 * gh1;
            gdt += (1.0f - lam) * inv * ds;
            glam -= dt * inv * ds;
            // what the predecessors pull from this point
            const float coef = (1.0f - lam) * dt / fnp;
            float np0 = al0 * gh0, np1 = al1 * gh1;
            float nq0 = coef * al0 * gh0, nq1 = coef * al1 * gh1;
            if (!hok) np0 = np1 = nq0 = nq1 = 0.0f;
            if (pa) {
                PO0[j] = np0; PO1[j] = np1; QO0[j] = nq0; QO1[j] = nq1;
            }
            ip0 = np0; ip1 = np1; iq0 = nq0; iq1 = nq1;
            // ---- stores
#pragma unroll
            for (int r = 0; r < RP; r++) {
                const int c = t * NR + r * N;
                if (pa && hok) {
                    const float2 vc = make_float2(x.dy[r] * ht0, x.dy[r] * ht1);
                    const float2 vb = make_float2(gbu0 * x.u[r], gbu1 * x.u[r]);
                    if constexpr (OVW) {
                        *(float2*)(dC + c) = vc;
                        *(float2*)(dB + c) = vb;
                    } else {
                        // one addition each (old + value): no read of the old value in the chain
                        atomicAdd(dC + c, vc.x);
                        atomicAdd(dC + c + 1, vc.y);
                        atomicAdd(dB + c, vb.x);
                        atomicAdd(dB + c + 1, vb.y);
                    }
                }
                float part = gbu0 * x.b[r].x + gbu1 * x.b[r].y;
                part = group_sum<GP>(part);
                if (pa && pl == 0) {
                    if (assign) du[t * R + r] = part;
                    else du[t * R + r] += part;
                }
            }
            gdt = group_sum<GP>(gdt);
            glam = group_sum<GP>(glam);
            if (pa && pl == 0) {
                if (assign) {
                    if (ddt) ddt[t] = gdt;
                    if (dlam) dlam[t] = glam;
                } else {
                    if (ddt) ddt[t] += gdt;
                    if (dlam) dlam[t] += glam;
                }
            }
            // the strip's leftmost processed column feeds the strip on the left
            if (q >= 0) { ob0 = ip0; ob1 = ip1; oq0 = iq0; oq1 = iq1; }
        }
        // ---- the last slot's output goes to warp w + 1 (row i - (SPW - 1))
        const int ro = i - (SPW - 1);
        if (w + 1 < nw && ro >= 0 && ro < H) {   // warp-uniform
            const int hs = ro & (BSB_K - 1);
            if (ro >= BSB_K && !mbar_wait(smem_u32(&hempty[(w + 1) * BSB_K + hs]), (uint32_t)(((ro / BSB_K) & 1) ^ 1))) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                return false;
            }
            if (ss == SPW - 1) {
                float* dst = hand + ((size_t)(w + 1) * BSB_K + hs) * 4 * GP;
                dst[pl] = ob0;
                dst[GP + pl] = ob1;
                dst[2 * GP + pl] = oq0;
                dst[3 * GP + pl] = oq1;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hfull[(w + 1) * BSB_K + hs]));
        }
        return true;
    };
    for (int i = 0; i < nsteps; i += 2) {
        if (!step(i, bufA, bufB)) return;
        if (i + 1 < nsteps && !step(i + 1, bufB, bufA)) return;
    }
    // ---- dA_log and dtheta partials of this CTA's pairs, in a fixed order
    red[threadIdx.x * 3 + 0] = gA0;
    red[threadIdx.x * 3 + 1] = gA1;
    red[threadIdx.x * 3 + 2] = gth;
    __syncthreads();
    if (threadIdx.x < GP) {
        float t0 = 0.0f, t1 = 0.0f, tt = 0.0f;
        for (int j = 0; j < nw * SPW; j++) {
            const int src = (j / SPW) * 32 + (j % SPW) * GP + threadIdx.x;
            t0 += red[src * 3 + 0];
            t1 += red[src * 3 + 1];
            tt += red[src * 3 + 2];
        }
        const int p = ln.g * GP + threadIdx.x;
        if (2 * p < N) g.pA[(long long)b * N + 2 * p] = t0;
        if (2 * p + 1 < N) g.pA[(long long)b * N + 2 * p + 1] = t1;
        if (p < 32) g.pth[(long long)b * 32 + p] = tt;
    }
}

// Forward for 2D grids, R in {1, 2, 4}, N even: the systolic strip pipeline of
// blockscan_bwd_strips run forwards (rows top to bottom, columns left to
// right), with the state pairs split into groups (CTA = (item, group of GP
// pairs)) so that an item runs on NG CTAs.  Strips of CW columns are numbered
// from the left; lane = (slot, pair), slot ss one row behind slot ss - 1.  The
// predecessor form R(theta) h and B*u of a point stays in registers for the
// next row (same column), moves along the strip in registers, to the next slot
// by a shuffle and to the next warp through mbarrier-guarded shared-memory
// slots (bounded waits).  Per point the arithmetic is blockscan_fwd_strips',
// so h and B*u are bit-identical to it; y is summed over the GP pairs of the
// group by shuffles and, with NG > 1, over the groups by bs_group_reduce in
// group order.
template <int RP>
struct BSFCol {
    float dt, lam, u[RP];
    float2 b[RP], c[RP];
};

template <typename T, int GP, int RP, int CW, bool FULL>
__global__ void __launch_bounds__(CW == 1 ? 512 : 256, 1) blockscan_fwd_gstrips(BSDesc s, int* status) {
    extern __shared__ __align__(16) unsigned char bsf_smem[];
    constexpr int SPW = 32 / GP;
    constexpr int R = RP;
    using Ln = BSLanes<GP>;
    const Ln ln(s);
    const int b = ln.b, n0 = ln.n0;
    const bool hok = FULL || ln.h0ok;   // FULL: N is a multiple of 2 GP, every lane has a pair
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int ss = ln.ps, pl = ln.pl;
    const int H = s.dims[0], W = s.dims[1];
    const int N = s.N, NR = N * R;
    const int nstrips = (W + CW - 1) / CW;
    const int st = w * SPW + ss;
    const int qa = st * CW;   // leftmost column of the strip
    const float A0 = hok ? s.A[n0] : 0.0f, A1 = hok ? s.A[n0 + 1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (hok) {
        kmb_cos_sin(s.theta[n0 >> 1], &cth, &sth);
    }
    const long long L = s.L;
    const T* __restrict__ u = (const T*)s.u + b * L * R;
    const T* __restrict__ dtp = (const T*)s.dt + b * L;
    const T* __restrict__ lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* __restrict__ Bp = (const T*)s.B + b * L * NR + n0;
    const T* __restrict__ Cp = (const T*)s.C + b * L * NR + n0;
    float* h = s.h + b * L * N + n0;
    float* Bu = s.Bu + b * L * N + n0;
    float* y = s.NG == 1 ? s.y + b * L * R : s.part + ((long long)ln.g * s.batch + b) * L * R;

    float* hand = (float*)bsf_smem;   // [nw][K][4][GP]
    uint64_t* hfull = (uint64_t*)(hand + (size_t)nw * BSB_K * 4 * GP);
    uint64_t* hempty = hfull + nw * BSB_K;
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw * BSB_K; i++) {
            mbar_init(smem_u32(&hfull[i]), 1);
            mbar_init(smem_u32(&hempty[i]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const float2 z2 = make_float2(0.0f, 0.0f);
    // rows and columns outside the grid (pipeline fill and drain, a partial last strip) are clamped
    // into it: their loads are valid and their results are never stored
    auto load_row = [&](BSFCol<RP>* c, int o) {
        o = min(max(o, 0), H - 1);
#pragma unroll
        for (int j = 0; j < CW; j++) {
            const int t = o * W + min(qa + j, W - 1);
            BSFCol<RP>& x = c[j];
            x.dt = ldv(dtp + t);
            x.lam = lamp ? ldv(lamp + t) : s.deflam;
            if constexpr (RP == 1) {
                x.u[0] = ldv(u + t);
            } else {
#pragma unroll
                for (int r = 0; r < RP; r += 2) {
                    const float2 u2 = ld2(u + t * R + r);
                    x.u[r] = u2.x;
                    x.u[r + 1] = u2.y;
                }
            }
#pragma unroll
            for (int r = 0; r < RP; r++) {
                x.b[r] = hok ? ld2(Bp + t * NR + r * N) : z2;
                x.c[r] = hok ? ld2(Cp + t * NR + r * N) : z2;
            }
        }
    };

    float rh0[CW], rh1[CW], rb0[CW], rb1[CW];   // previous row of this strip's columns: R(theta) h, B*u
#pragma unroll
    for (int j = 0; j < CW; j++) rh0[j] = rh1[j] = rb0[j] = rb1[j] = 0.0f;
    float ob0 = 0.0f, ob1 = 0.0f, oc0 = 0.0f, oc1 = 0.0f;   // this slot's output to the strip on its right
    // two row buffers used in turn (no register copy that would wait for the prefetch to land)
    BSFCol<RP> bufA[CW], bufB[CW];
    load_row(bufA, -ss);
    const int nsteps = H + SPW - 1;
    auto step = [&](const int i, BSFCol<RP>* cur, BSFCol<RP>* nxt) -> bool {
        const int o = i - ss;
        const bool act = st < nstrips && o >= 0 && o < H;
        load_row(nxt, o + 1);
        // ---- inner predecessor of the leftmost column: the strip on the left, same row
        float lh0 = __shfl_up_sync(0xffffffffu, ob0, GP);
        float lh1 = __shfl_up_sync(0xffffffffu, ob1, GP);
        float lb0 = __shfl_up_sync(0xffffffffu, oc0, GP);
        float lb1 = __shfl_up_sync(0xffffffffu, oc1, GP);
        if (ss == 0) lh0 = lh1 = lb0 = lb1 = 0.0f;
        if (w > 0 && i < H) {   // warp-uniform: slot 0 takes row i of warp w - 1's last strip
            const int hs = i & (BSB_K - 1);
            if (!mbar_wait(smem_u32(&hfull[w * BSB_K + hs]), (uint32_t)((i / BSB_K) & 1))) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                return false;
            }
            if (ss == 0) {
                const float* src = hand + ((size_t)w * BSB_K + hs) * 4 * GP;
                lh0 = src[pl];
                lh1 = src[GP + pl];
                lb0 = src[2 * GP + pl];
                lb1 = src[3 * GP + pl];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hempty[w * BSB_K + hs]));
        }
#pragma unroll
        for (int j = 0; j < CW; j++) {
            const int q = qa + j;
            const bool pa = act && q < W;
            const BSFCol<RP>& x = cur[j];
            const int t = pa ? o * W + q : 0;
            const float dt = x.dt, lam = x.lam;
            float bu0 = 0.0f, bu1 = 0.0f;
#pragma unroll
            for (int r = 0; r < RP; r++) {
                bu0 = __fmaf_rn(x.b[r].x, x.u[r], bu0);
                bu1 = __fmaf_rn(x.b[r].y, x.u[r], bu1);
            }
            const float al0 = kmb_exp(dt * A0, s.fast), al1 = kmb_exp(dt * A1, s.fast);
            float hn0 = 0.0f, hn1 = 0.0f, bacc0 = 0.0f, bacc1 = 0.0f;
            int np = 0;
            if (o > 0) {   // outer predecessor (o-1, q): this column's previous row
                hn0 = __fmaf_rn(al0, rh0[j], hn0);
                hn1 = __fmaf_rn(al1, rh1[j], hn1);
                bacc0 += rb0[j];
                bacc1 += rb1[j];
                np++;
            }
            if (q > 0) {   // inner predecessor (o, q-1): the previous column of this row
                hn0 = __fmaf_rn(al0, lh0, hn0);
                hn1 = __fmaf_rn(al1, lh1, hn1);
                bacc0 += lb0;
                bacc1 += lb1;
                np++;
            }
            if (np > 0) {
                const float bs = (1.0f - lam) * dt / (float)np;
                hn0 = __fmaf_rn(bs * al0, bacc0, hn0);
                hn1 = __fmaf_rn(bs * al1, bacc1, hn1);
            }
            const float gm = lam * dt;
            hn0 = __fmaf_rn(gm, bu0, hn0);
            hn1 = __fmaf_rn(gm, bu1, hn1);
            if (pa && hok) {
                *(float2*)(h + t * N) = make_float2(hn0, hn1);
                *(float2*)(Bu + t * N) = make_float2(bu0, bu1);
            }
            const float r0 = cth * hn0 - sth * hn1, r1 = sth * hn0 + cth * hn1;
            if (pa) {
                rh0[j] = r0; rh1[j] = r1; rb0[j] = bu0; rb1[j] = bu1;
            }
            lh0 = r0; lh1 = r1; lb0 = bu0; lb1 = bu1;
            if (q < W) { ob0 = r0; ob1 = r1; oc0 = bu0; oc1 = bu1; }
#pragma unroll
            for (int r = 0; r < RP; r++) {
                float part = x.c[r].x * hn0;
                part = __fmaf_rn(x.c[r].y, hn1, part);
                part = group_sum<GP>(hok ? part : 0.0f);
                if (pa && pl == 0) y[t * R + r] = part;
            }
        }
        // ---- the last slot's output goes to warp w + 1 (row i - (SPW - 1))
        const int ro = i - (SPW - 1);
        if (w + 1 < nw && ro >= 0 && ro < H) {   // warp-uniform
            const int hs = ro & (BSB_K - 1);
            if (ro >= BSB_K &&
                !mbar_wait(smem_u32(&hempty[(w + 1) * BSB_K + hs]), (uint32_t)(((ro / BSB_K) & 1) ^ 1))) {
                set_status(status, KMB_ERR_TIMEOUT_Y);
                return false;
            }
            if (ss == SPW - 1) {
                float* dst = hand + ((size_t)(w + 1) * BSB_K + hs) * 4 * GP;
                dst[pl] = ob0;
                dst[GP + pl] = ob1;
                dst[2 * GP + pl] = oc0;
                dst[3 * GP + pl] = oc1;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hfull[(w + 1) * BSB_K + hs]));
        }
        return true;
    };
    for (int i = 0; i < nsteps; i += 2) {
        if (!step(i, bufA, bufB)) return;
        if (i + 1 < nsteps && !step(i + 1, bufB, bufA)) return;
    }
}

// out[i] (+)= sum_g part[g * n + i], g = 0 .. NG-1 in order
__global__ void bs_group_reduce(const float* __restrict__ part, float* __restrict__ out, long long n, int ng,
                                int accumulate) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float acc = 0.0f;
    for (int j = 0; j < ng; j++) acc += part[(long long)j * n + i];
    out[i] = accumulate ? out[i] + acc : acc;
}

// out[i] += sum_j part[j*stride + i]
__global__ void bs_reduce_add(const float* __restrict__ part, float* __restrict__ out, int count, long long n,
                              long long stride) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float acc = 0.0f;
    for (long long j = 0; j < n; j++) acc += part[j * stride + i];
    out[i] += acc;
}

}  // namespace kmb

// ------------------------------------------------------------------ host side
#include <algorithm>
#include <cstring>
#include <map>
#include <vector>
#include "../../include/wavefront_plan.h"

namespace kmb {
void* workspace(int slot, size_t bytes);
int set_error(const char* msg);
int set_cuda_error(const char* where, cudaError_t e);
enum { WS_BS_FWD = 3, WS_BS_SCRATCH = 4 };
int* device_status();
// forward choice of this host thread (kmb_blockscan_set_strips modes 0-3) and the path of the last forward
static thread_local int tl_bs_mode = 1, tl_bs_no_strips = 0, tl_bs_no_staging = 0, tl_bs_path = -1;
// backward choice (1: strips where the shape allows, 0: level kernels) and the path of the last backward
static thread_local int tl_bs_bwd_strips = 1, tl_bs_bwd_path = -1;

// Device copy of the wavefront plan of `dims` (level starts [nlev + 1], then the
// points of every level [L]), cached per host thread, device and shape.
// Shared with the Scan-A backward (scannd_bwd.cu).
struct PlanEntry {
    int nlev = 0, wmax = 0;
    int* dev = nullptr;
};
static thread_local std::map<int, std::map<std::vector<long>, PlanEntry>> tl_plans;

// Device layout: level starts [nlev + 1] | points of every level [L] | position
// of every point inside its level [L] | neighbour mask of every point [L]
// (bit k: a predecessor along axis k, bit 8 + k: a successor along axis k).
int device_plan_ex(const std::vector<long>& dims, long L, int** out, int* nlev, int* wmax, cudaStream_t st) {
    int devid = 0;
    cudaGetDevice(&devid);
    PlanEntry& pe = tl_plans[devid][dims];
    if (!pe.dev) {
        KMWavefrontPlan* pl = km_wavefront_plan_create(dims.data(), (long)dims.size(), 0);
        if (!pl) return set_error("cannot build the wavefront plan");
        const int nl = (int)pl->max_level + 1;
        std::vector<int> host(nl + 1 + 3 * (size_t)L);
        int* starts = host.data();
        int* pts = starts + nl + 1;
        int* pos = pts + L;
        int* mask = pos + L;
        int wm = 0;
        for (int i = 0; i <= nl; i++) starts[i] = (int)pl->level_starts[i];
        for (int l = 0; l < nl; l++) {
            wm = std::max(wm, starts[l + 1] - starts[l]);
            for (int i = starts[l]; i < starts[l + 1]; i++) {
                pts[i] = (int)pl->level_offsets[i];
                pos[pts[i]] = i - starts[l];
            }
        }
        km_wavefront_plan_free(pl);
        const int nd = (int)dims.size();
        for (long t = 0; t < L; t++) {
            long rem = t;
            int m = 0;
            for (int k = nd - 1; k >= 0; k--) {
                const long ik = rem % dims[k];
                rem /= dims[k];
                if (ik > 0) m |= 1 << k;
                if (ik < dims[k] - 1) m |= 1 << (8 + k);
            }
            mask[t] = m;
        }
        int* d = nullptr;
        cudaError_t e = cudaMalloc(&d, host.size() * sizeof(int));  // one allocation per shape, kept for reuse
        if (e != cudaSuccess) return set_cuda_error("plan allocation", e);
        e = cudaMemcpyAsync(d, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // the host vector goes out of scope
        if (e != cudaSuccess) {
            cudaFree(d);
            return set_cuda_error("plan upload", e);
        }
        pe.dev = d;
        pe.nlev = nl;
        pe.wmax = wm;
    }
    *out = pe.dev;
    *nlev = pe.nlev;
    if (wmax) *wmax = pe.wmax;
    return 0;
}

int device_plan(const std::vector<long>& dims, long L, int** out, int* nlev, cudaStream_t st) {
    return device_plan_ex(dims, L, out, nlev, nullptr, st);
}

static int bs_desc(const KMBlockScanParams* p, long batch, BSDesc* s, cudaStream_t st) {
    if (!p || batch < 1 || p->N < 1 || p->N > 64 || p->R < 1 || p->R > 64 || p->L < 1 || !p->u || !p->dt ||
        !p->B || !p->C || !p->A_log || !p->h || !p->Bu || !p->y)
        return set_error("invalid KMBlockScanParams (N must be 1..64)");
    if (p->N >= 2 && !p->theta) return set_error("KMBlockScanParams: theta is required (RoPE is always on)");
    std::vector<long> dims;
    if (p->ndims <= 1) {
        dims.push_back(p->L);
    } else {
        if (p->ndims > BS_MAXND || !p->dims) return set_error("blockscan: ndims must be <= 8");
        long prod = 1;
        for (long i = 0; i < p->ndims; i++) {
            if (p->dims[i] <= 0) return set_error("blockscan: invalid dims");
            dims.push_back(p->dims[i]);
            prod *= p->dims[i];
        }
        if (prod != p->L) return set_error("blockscan: product of dims != L");
    }
    if (p->L > 0x7fffffffL || (long long)p->L * p->N * p->R >= (1LL << 31))
        return set_error("blockscan: L * N * R must be below 2^31 per item (32-bit indexing inside an item)");
    memset(s, 0, sizeof(*s));
    s->nd = p->ndims <= 1 ? 1 : (int)p->ndims;
    s->N = (int)p->N;
    s->R = (int)p->R;
    s->P2 = (s->N + 1) / 2;
    s->GP = 1;
    while (s->GP < 8 && s->GP < s->P2) s->GP *= 2;
    s->NG = (s->P2 + s->GP - 1) / s->GP;
    s->fast = p->use_fast_exp != 0;
    s->deflam = p->default_lambda;
    s->L = p->L;
    s->batch = batch;
    int stv = 1;
    for (int a = (int)dims.size() - 1; a >= 0; a--) {
        s->dims[a] = (int)dims[a];
        s->strides[a] = stv;
        stv *= (int)dims[a];
    }
    if (p->ndims <= 1) s->nd = 1;
    int* plan = nullptr;
    if (device_plan_ex(dims, p->L, &plan, &s->nlev, &s->wmax, st)) return -1;
    s->lev_start = plan;
    s->lev_pts = plan + s->nlev + 1;
    s->lev_pos = s->lev_pts + p->L;
    s->nbr = s->lev_pos + p->L;
    s->bf16 = p->inputs_bf16 != 0;
    s->u = p->u; s->dt = p->dt; s->lam = p->lambda; s->B = p->B; s->C = p->C; s->A = p->A_log;
    s->theta = p->theta; s->h = p->h; s->Bu = p->Bu; s->y = p->y;
    return 0;
}

static int bs_threads(const BSDesc& s) {
    // widest level decides how many warps can work at once
    long long w = 1;
    for (int k = 0; k < s.nd; k++) w *= s.dims[k];
    if (s.nd == 1) return 32;
    return 512;
}

// shared memory of the ring kernels (two levels of GP pairs, two arrays)
static size_t ring_bytes(const BSDesc& s) { return (size_t)2 * 2 * s.wmax * s.GP * 2 * sizeof(float); }
static bool ring_ok(const BSDesc& s) { return s.nd <= 3 && s.R <= 4 && ring_bytes(s) <= 200 * 1024; }

template <typename T, int GP, int RM>
static void bs_fwd_ring_r(const BSDesc& s, cudaStream_t st) {
    const dim3 grid((unsigned)(s.batch * s.NG));
    const int th = bs_threads(s);
    const size_t sm = ring_bytes(s);
    auto go = [&](auto kern) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        kern<<<grid, th, sm, st>>>(s);
    };
    if (s.nd <= 1) go(blockscan_fwd_ring<T, GP, RM, 1>);
    else if (s.nd == 2) go(blockscan_fwd_ring<T, GP, RM, 2>);
    else go(blockscan_fwd_ring<T, GP, RM, 3>);
}

template <typename T, int GP>
static void bs_fwd_launch(const BSDesc& s, cudaStream_t st) {
    const dim3 grid((unsigned)(s.batch * s.NG));
    const int th = bs_threads(s);
    if (ring_ok(s)) {
        if (s.R <= 1) bs_fwd_ring_r<T, GP, 1>(s, st);
        else if (s.R <= 2) bs_fwd_ring_r<T, GP, 2>(s, st);
        else bs_fwd_ring_r<T, GP, 4>(s, st);
        return;
    }
    if (s.R <= 1) blockscan_fwd_kernel<T, GP, 1><<<grid, th, 0, st>>>(s);
    else if (s.R <= 2) blockscan_fwd_kernel<T, GP, 2><<<grid, th, 0, st>>>(s);
    else if (s.R <= 4) blockscan_fwd_kernel<T, GP, 4><<<grid, th, 0, st>>>(s);
    else blockscan_fwd_kernel<T, GP, 0><<<grid, th, 0, st>>>(s);
}
template <typename T, int GP, int RM>
static void bs_bwd_launch_r(const BSDesc& s, const BSGrad& g, cudaStream_t st) {
    const dim3 grid((unsigned)(s.batch * s.NG));
    const int th = bs_threads(s);
    if (s.nd <= 1) blockscan_bwd_kernel<T, GP, RM, 1><<<grid, th, 0, st>>>(s, g);
    else if (s.nd == 2) blockscan_bwd_kernel<T, GP, RM, 2><<<grid, th, 0, st>>>(s, g);
    else if (s.nd == 3) blockscan_bwd_kernel<T, GP, RM, 3><<<grid, th, 0, st>>>(s, g);
    else blockscan_bwd_generic<T, GP><<<grid, th, 0, st>>>(s, g);
}
template <typename T, int GP>
static void bs_bwd_launch(const BSDesc& s, const BSGrad& g, cudaStream_t st) {
    if (s.R <= 1) bs_bwd_launch_r<T, GP, 1>(s, g, st);
    else if (s.R <= 2) bs_bwd_launch_r<T, GP, 2>(s, g, st);
    else if (s.R <= 4) bs_bwd_launch_r<T, GP, 4>(s, g, st);
    else blockscan_bwd_generic<T, GP><<<(unsigned)(s.batch * s.NG), bs_threads(s), 0, st>>>(s, g);
}
template <typename T>
static void bs_fwd_dispatch(const BSDesc& s, cudaStream_t st) {
    switch (s.GP) {
        case 1: bs_fwd_launch<T, 1>(s, st); break;
        case 2: bs_fwd_launch<T, 2>(s, st); break;
        case 4: bs_fwd_launch<T, 4>(s, st); break;
        default: bs_fwd_launch<T, 8>(s, st); break;
    }
}
template <typename T>
static void bs_bwd_dispatch(const BSDesc& s, const BSGrad& g, cudaStream_t st) {
    switch (s.GP) {
        case 1: bs_bwd_launch<T, 1>(s, g, st); break;
        case 2: bs_bwd_launch<T, 2>(s, g, st); break;
        case 4: bs_bwd_launch<T, 4>(s, g, st); break;
        default: bs_bwd_launch<T, 8>(s, g, st); break;
    }
}
// The systolic backward for 2D grids, R in {1, 2, 4}, N even, when the strips fit in 8 warps.  false: not taken.
constexpr int BSB_CW = 2;   // columns per strip (4 measured slower: fewer warps, longer serial steps)
static bool bs_bwd_strips_launch(const BSDesc& s, const BSGrad& g, cudaStream_t st) {
    if (!tl_bs_bwd_strips || s.nd != 2 || !(s.R == 1 || s.R == 2 || s.R == 4) || s.N % 2) return false;
    const int spw = 32 / s.GP;
    const int nstrips = (s.dims[1] + BSB_CW - 1) / BSB_CW;
    const int nw = (nstrips + spw - 1) / spw;
    if (nw > 8) return false;
    int* status = device_status();
    if (!status) return false;
    const size_t sm = (size_t)nw * BSB_K * 4 * s.GP * sizeof(float) + 2 * nw * BSB_K * sizeof(uint64_t) +
                      (size_t)nw * 32 * 3 * sizeof(float);
    const dim3 grid((unsigned)(s.batch * s.NG));
    auto go = [&](auto kern) { kern<<<grid, nw * 32, sm, st>>>(s, g, status); };
#define KMB_BSB_O(TT, GPV, RV, FL)                                                    \
    do {                                                                            \
        if (g.overwrite) go(blockscan_bwd_strips<TT, GPV, RV, BSB_CW, true, FL>);   \
        else go(blockscan_bwd_strips<TT, GPV, RV, BSB_CW, false, FL>);              \
    } while (0)
#define KMB_BSB_R(TT, GPV, FL)                                \
    do {                                                    \
        if (s.R == 1) KMB_BSB_O(TT, GPV, 1, FL);             \
        else if (s.R == 2) KMB_BSB_O(TT, GPV, 2, FL);        \
        else KMB_BSB_O(TT, GPV, 4, FL);                      \
    } while (0)
#define KMB_BSB_GP(TT)                          \
    do {                                        \
        switch (s.GP) {                         \
            case 1: KMB_BSB_R(TT, 1, false); break;                       \
            case 2: KMB_BSB_R(TT, 2, false); break;                       \
            case 4: KMB_BSB_R(TT, 4, false); break;                       \
            default:                                                        \
                if (s.N % 16 == 0) KMB_BSB_R(TT, 8, true);                \
                else KMB_BSB_R(TT, 8, false);                             \
                break;                                                      \
        }                                       \
    } while (0)
    if (s.bf16) KMB_BSB_GP(__nv_bfloat16);
    else KMB_BSB_GP(float);
#undef KMB_BSB_GP
#undef KMB_BSB_R
#undef KMB_BSB_O
    tl_bs_bwd_path = 1;
    return true;
}

// The grouped strip forward for 2D grids, R in {1, 2, 4}, N even, when the strips fit in 8 warps.
// columns per forward strip (one column, in 16-warp CTAs, measured 1 % slower per block step)
constexpr int BSF_CW = 2;
static bool bs_fwd_gstrips_launch(const BSDesc& s, cudaStream_t st) {
    if (tl_bs_mode != 1 || s.nd != 2 || !(s.R == 1 || s.R == 2 || s.R == 4) || s.N % 2) return false;
    const int spw = 32 / s.GP;
    const int nstrips = (s.dims[1] + BSF_CW - 1) / BSF_CW;
    const int nw = (nstrips + spw - 1) / spw;
    if (nw > (BSF_CW == 1 ? 16 : 8)) return false;
    int* status = device_status();
    if (!status) return false;
    const size_t sm = (size_t)nw * BSB_K * 4 * s.GP * sizeof(float) + 2 * nw * BSB_K * sizeof(uint64_t);
    const dim3 grid((unsigned)(s.batch * s.NG));
    auto go = [&](auto kern) { kern<<<grid, nw * 32, sm, st>>>(s, status); };
#define KMB_BSF_R(TT, GPV, FL)                                                  \
    do {                                                                      \
        if (s.R == 1) go(blockscan_fwd_gstrips<TT, GPV, 1, BSF_CW, FL>);      \
        else if (s.R == 2) go(blockscan_fwd_gstrips<TT, GPV, 2, BSF_CW, FL>); \
        else go(blockscan_fwd_gstrips<TT, GPV, 4, BSF_CW, FL>);               \
    } while (0)
#define KMB_BSF_GP(TT)                          \
    do {                                        \
        switch (s.GP) {                         \
            case 1: KMB_BSF_R(TT, 1, false); break;                       \
            case 2: KMB_BSF_R(TT, 2, false); break;                       \
            case 4: KMB_BSF_R(TT, 4, false); break;                       \
            default:                                                        \
                if (s.N % 16 == 0) KMB_BSF_R(TT, 8, true);                \
                else KMB_BSF_R(TT, 8, false);                             \
                break;                                                      \
        }                                       \
    } while (0)
    if (s.bf16) KMB_BSF_GP(__nv_bfloat16);
    else KMB_BSF_GP(float);
#undef KMB_BSF_GP
#undef KMB_BSF_R
    return true;
}

static void group_reduce(const float* part, float* out, long long n, int ng, int accumulate, cudaStream_t st) {
    bs_group_reduce<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, out, n, ng, accumulate);
}

}  // namespace kmb

using namespace kmb;

extern "C" void kmb_blockscan_set_strips(int mode) {
    tl_bs_mode = mode;
    tl_bs_no_strips = mode == 0 ? 1 : 0;
    tl_bs_no_staging = mode == 2 ? 1 : 0;
}
extern "C" int kmb_blockscan_last_forward_path(void) { return tl_bs_path; }
extern "C" void kmb_blockscan_set_backward_strips(int on) { tl_bs_bwd_strips = on ? 1 : 0; }
extern "C" int kmb_blockscan_last_backward_path(void) { return tl_bs_bwd_path; }

extern "C" int kmb_blockscan_forward(const KMBlockScanParams* p, long batch, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    BSDesc s;
    if (bs_desc(p, batch, &s, st)) return -1;
    const long long ny = (long long)batch * s.L * s.R;
    if (s.NG > 1) {
        s.part = (float*)workspace(WS_BS_FWD, (size_t)s.NG * ny * sizeof(float));
        if (!s.part) return set_error("workspace allocation failed");
    }
    // 2D grids, N even: the grouped systolic strip kernel (NG CTAs per item)
    if (bs_fwd_gstrips_launch(s, st)) {
        tl_bs_path = 3;
        if (s.NG > 1) group_reduce(s.part, s.y, ny, s.NG, 0, st);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? 0 : set_cuda_error("blockscan_fwd_gstrips", e);
    }
    // 2D grids with an inner extent <= 64: the systolic strip kernel (one CTA per item)
    if (s.nd == 2 && s.dims[1] <= 64 && s.N <= 64 && (s.R == 1 || s.R == 2 || s.R == 4) && !tl_bs_no_strips) {
        int* status = device_status();
        if (status) {
            const int S = (s.dims[1] + BSS_WC - 1) / BSS_WC;
            const int sb = s.bf16 ? BSStage<__nv_bfloat16>(s.R, s.N, s.lam != nullptr).bytes
                                  : BSStage<float>(s.R, s.N, s.lam != nullptr).bytes;
            const size_t sm_base =
                (size_t)S * BSS_K * 4 * 32 * sizeof(float) + (2 * S * BSS_K + S * BSS_NSS) * sizeof(uint64_t);
            const size_t sm_staged = sm_base + 128 + (size_t)S * BSS_NSS * sb;   // + alignment of the stages
            // staged rows (bulk copies of whole 16-byte pieces) when every strip is full, N % 8 == 0
            // and the stages fit
            const bool staged = s.dims[1] % BSS_WC == 0 && s.N % 8 == 0 && !tl_bs_no_staging &&
                                sm_staged <= 200 * 1024;
            const size_t sm = staged ? sm_staged : sm_base;
            auto go = [&](auto kern) {
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
                kern<<<(unsigned)batch, S * 32, sm, st>>>(s, status);
            };
#define KMB_BSS_GO(TT, ST)                                              \
    do {                                                                \
        if (s.R == 1) go(blockscan_fwd_strips<TT, 1, ST>);              \
        else if (s.R == 2) go(blockscan_fwd_strips<TT, 2, ST>);         \
        else go(blockscan_fwd_strips<TT, 4, ST>);                       \
    } while (0)
            if (s.bf16) {
                if (staged) KMB_BSS_GO(__nv_bfloat16, true);
                else KMB_BSS_GO(__nv_bfloat16, false);
            } else {
                if (staged) KMB_BSS_GO(float, true);
                else KMB_BSS_GO(float, false);
            }
#undef KMB_BSS_GO
            tl_bs_path = staged ? 2 : 1;
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? 0 : set_cuda_error("blockscan_fwd_strips", e);
        }
    }
    tl_bs_path = 0;
    if (s.bf16) bs_fwd_dispatch<__nv_bfloat16>(s, st);
    else bs_fwd_dispatch<float>(s, st);
    if (s.NG > 1) group_reduce(s.part, s.y, ny, s.NG, 0, st);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("blockscan_fwd", e);
}

extern "C" int kmb_blockscan_backward_ex(const KMBlockScanParams* p, long batch, const float* dy,
                                         const KMBlockScanGrads* gr, int overwrite, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (!dy || !gr || !gr->dB || !gr->dC || !gr->du) return set_error("blockscan backward: dy, dB, dC, du required");
    BSDesc s;
    if (bs_desc(p, batch, &s, st)) return -1;
    const size_t nG = (size_t)batch * s.L * s.N;
    const size_t ny = (size_t)batch * s.L * s.R, nl = (size_t)batch * s.L;
    const size_t npart = s.NG > 1 ? (size_t)s.NG * (ny + 2 * nl) : 0;
    const size_t bytes = (nG + (size_t)batch * s.N + (size_t)batch * 32 + npart) * sizeof(float) + 512;
    char* w = (char*)workspace(WS_BS_SCRATCH, bytes);
    if (!w) return set_error("workspace allocation failed");
    BSGrad g;
    g.dy = dy;
    g.dB = gr->dB; g.dC = gr->dC; g.du = gr->du; g.ddt = gr->ddt; g.dlam = gr->dlambda;
    g.G = (float*)w;
    g.pA = g.G + nG;
    g.pth = g.pA + (size_t)batch * s.N;
    g.pdu = g.pth + (size_t)batch * 32;
    g.pddt = g.pdu + (size_t)s.NG * ny;
    g.pdlam = g.pddt + (size_t)s.NG * nl;
    g.overwrite = overwrite ? 1 : 0;
    if (!bs_bwd_strips_launch(s, g, st)) {
        tl_bs_bwd_path = 0;
        if (overwrite) {   // the level kernels accumulate: clear the outputs first
            cudaError_t e = cudaSuccess;
            const size_t nbc = ny * s.N * sizeof(float);
            if (e == cudaSuccess) e = cudaMemsetAsync(gr->dB, 0, nbc, st);
            if (e == cudaSuccess) e = cudaMemsetAsync(gr->dC, 0, nbc, st);
            if (e == cudaSuccess) e = cudaMemsetAsync(gr->du, 0, ny * sizeof(float), st);
            if (e == cudaSuccess && gr->ddt) e = cudaMemsetAsync(gr->ddt, 0, nl * sizeof(float), st);
            if (e == cudaSuccess && gr->dlambda) e = cudaMemsetAsync(gr->dlambda, 0, nl * sizeof(float), st);
            if (e != cudaSuccess) return set_cuda_error("blockscan backward memset", e);
            g.overwrite = 0;
        }
        if (s.bf16) bs_bwd_dispatch<__nv_bfloat16>(s, g, st);
        else bs_bwd_dispatch<float>(s, g, st);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("blockscan_bwd", e);
    if (s.NG > 1) {
        const int acc = g.overwrite ? 0 : 1;
        group_reduce(g.pdu, gr->du, (long long)ny, s.NG, acc, st);
        if (gr->ddt) group_reduce(g.pddt, gr->ddt, (long long)nl, s.NG, acc, st);
        if (gr->dlambda) group_reduce(g.pdlam, gr->dlambda, (long long)nl, s.NG, acc, st);
    }
    if (gr->dA_log) bs_reduce_add<<<1, 64, 0, st>>>(g.pA, gr->dA_log, s.N, batch, s.N);
    if (gr->dtheta && s.N >= 2) bs_reduce_add<<<1, 32, 0, st>>>(g.pth, gr->dtheta, s.N / 2, batch, 32);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("blockscan reduce", e);
}

extern "C" int kmb_blockscan_backward(const KMBlockScanParams* p, long batch, const float* dy,
                                      const KMBlockScanGrads* gr, void* stream) {
    return kmb_blockscan_backward_ex(p, batch, dy, gr, 0, stream);
}
