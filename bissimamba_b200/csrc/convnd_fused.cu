// convnd_fused.cu -- depthwise causal convND forward + backward in one launch
// (reference src/convnd.c:396-531): ndims <= 2 with K <= 4
// and D a multiple of 8 on the kernel below; ndims = 3 with K <= 3 and D a
// multiple of 4 on the streaming 3D kernel further down.
//
// A CTA owns (item b, slab of T0 planes of the outermost axis, 8 channels).
// It stages the input slab with its K-1 causal halo planes / rows / columns
// on the low side, and the dy slab with the halo on the high side, into
// shared memory, zero-padded, so no tap needs a bounds test.  Then each
// thread walks runs of R consecutive points along the innermost axis for one
// float4 of channels:
//   forward  out[x]  = bias + sum_k in[x - s_k] ker[k]   (taps in ascending
//            kernel-linear order, the reference's order: bit-identical)
//   dinput   din[x]  = sum_k dy[x + s_k] ker[k]          (gather, no atomics)
//   dkernel  acc[k] += dy[x] in[x - s_k]                  (per-CTA partials)
// A row of R + K - 1 values along the innermost axis serves all K taps of that
// axis for the R points, so shared-memory reads per point fall from K^nd to
// K^(nd-1) (R + K - 1) / R.  The input values read for the forward are the
// ones the dkernel products need, so they are read once for both.  The
// per-CTA dkernel / dbias partials are summed over the CTA in a fixed order
// and written to part[(b * nslab + slab)][V + 1][D]; a second launch adds the
// chunks in order (deterministic).  Global traffic: input and dy read once
// (plus the halo planes of the next slab), out and dinput written once.
#include "kmb_common.cuh"
#include "kmb_sync.cuh"

namespace kmb {

constexpr int CF_THREADS = 256;
constexpr int CF_SMEM_MAX = 110 * 1024;   // two CTAs per SM

struct FusedGeom {
    int T0, nslab;              // planes of axis 0 per slab, slabs per item
    int pd[3];                  // padded extents of the slab (axis 0 includes the K - 1 halo planes)
    int ps[3];                  // padded strides (in points)
    int slab_pts;               // points of one padded slab
    int slab_slots;             // point slots allocated (one spare slot after every 4 points)
};

template <int ND, int K>
struct CfTaps {
    static constexpr int V = ND == 1 ? K : (ND == 2 ? K * K : K * K * K);
    static constexpr int ROWS = V / K;   // taps of the outer axes: one shared-memory row each
};

// N channels per thread (1, 2 or 4 floats)
template <int N> struct CfVec;
template <> struct CfVec<4> { using T = float4; };
template <> struct CfVec<2> { using T = float2; };
template <> struct CfVec<1> { using T = float; };
// packed fp32 pairs: per component exactly __fmaf_rn / __fadd_rn, two channels per instruction
__device__ __forceinline__ void cf_fma(float4& a, const float4 x, const float4 y) {
    const float2 lo = __ffma2_rn(make_float2(x.x, x.y), make_float2(y.x, y.y), make_float2(a.x, a.y));
    const float2 hi = __ffma2_rn(make_float2(x.z, x.w), make_float2(y.z, y.w), make_float2(a.z, a.w));
    a = make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ void cf_fma(float2& a, const float2 x, const float2 y) { a = __ffma2_rn(x, y, a); }
__device__ __forceinline__ void cf_fma(float& a, const float x, const float y) { a = __fmaf_rn(x, y, a); }
__device__ __forceinline__ void cf_add(float4& a, const float4 x) {
    const float2 lo = __fadd2_rn(make_float2(a.x, a.y), make_float2(x.x, x.y));
    const float2 hi = __fadd2_rn(make_float2(a.z, a.w), make_float2(x.z, x.w));
    a = make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ void cf_add(float2& a, const float2 x) { a = __fadd2_rn(a, x); }
__device__ __forceinline__ void cf_add(float& a, const float x) { a += x; }
template <typename V> __device__ __forceinline__ V cf_zero();
template <> __device__ __forceinline__ float4 cf_zero<float4>() { return make_float4(0.f, 0.f, 0.f, 0.f); }
template <> __device__ __forceinline__ float2 cf_zero<float2>() { return make_float2(0.f, 0.f); }
template <> __device__ __forceinline__ float cf_zero<float>() { return 0.0f; }
__device__ __forceinline__ float4 cf_shfl(float4 v, int o) {
    return make_float4(__shfl_xor_sync(~0u, v.x, o), __shfl_xor_sync(~0u, v.y, o), __shfl_xor_sync(~0u, v.z, o),
                       __shfl_xor_sync(~0u, v.w, o));
}
__device__ __forceinline__ float2 cf_shfl(float2 v, int o) {
    return make_float2(__shfl_xor_sync(~0u, v.x, o), __shfl_xor_sync(~0u, v.y, o));
}
__device__ __forceinline__ float cf_shfl(float v, int o) { return __shfl_xor_sync(~0u, v, o); }

// Shared-memory slot of padded point pt: one spare slot after every four points,
// so the runs of four points that the threads of a warp read start in different
// banks (no conflicts for 4-, 8- or 16-byte reads).
__device__ __forceinline__ int cf_slot(int pt) { return pt + (pt >> 2); }

// MODE bit 0: forward (out); bit 1: backward (dinput, dkernel / dbias partials).
// CG float4 channel lanes (4 CG channels) per CTA; N channels per thread.
template <int ND, int K, int R, int MODE, int N, int CG>
__global__ void __launch_bounds__(CF_THREADS, 2) conv_fused_kernel(ConvDesc c, FusedGeom g,
                                                                   const float4* __restrict__ in,
                                                                   const float* __restrict__ ker,
                                                                   const float* __restrict__ bias,
                                                                   const float4* __restrict__ dy,
                                                                   float* __restrict__ out, float* __restrict__ din,
                                                                   float* __restrict__ part) {
    using T = CfTaps<ND, K>;
    using V = typename CfVec<N>::T;
    constexpr bool FWD = MODE & 1, BWD = (MODE & 2) != 0;
    constexpr int NL = CG * 4 / N;                           // threads per point (channel lanes of N)
    constexpr int H = K - 1;
    extern __shared__ __align__(16) float4 cf_smem[];
    float4* sIN = cf_smem;                                   // [slot][CG]
    float4* sDY = cf_smem + g.slab_slots * CG;
    const int D4 = c.D >> 2;
    const int slab = blockIdx.x % g.nslab;
    const long long b = blockIdx.x / g.nslab;
    const int lane0 = blockIdx.y * CG;                       // first float4 channel lane of this CTA
    const int z0 = slab * g.T0;
    const int dims0 = (int)c.dims[0];
    const int nz = min(g.T0, dims0 - z0);                    // planes this CTA produces
    const int d1 = ND > 1 ? (int)c.dims[ND > 1 ? 1 : 0] : 1;
    const int d2 = ND > 2 ? (int)c.dims[ND > 2 ? 2 : 0] : 1;
    const long long ibase = b * c.P;                         // item base in points
    const int tid = threadIdx.x, wl = tid & 31, warp = tid >> 5;

    // ---- stage the slabs, one padded row of the innermost axis at a time (zero halo):
    // padded (pz, py, px) <- input (z0 + pz - H, py - H, px - H) and dy (z0 + pz, py, px)
    {
        const int pdl = g.pd[ND - 1];                        // padded innermost extent
        const int nrows = g.slab_pts / pdl;
        const int dl_ = ND == 1 ? dims0 : (ND == 2 ? d1 : d2);
        for (int row = warp; row < nrows; row += CF_THREADS / 32) {
            int c0 = row, c1 = 0;
            if (ND == 3) {
                c0 = row / g.pd[1];
                c1 = row - c0 * g.pd[1];
            }
            // source row coordinates (outer axes) for the input and for dy
            const int si0 = ND == 1 ? 0 : z0 + c0 - H, si1 = c1 - H;
            const int sd0 = ND == 1 ? 0 : z0 + c0, sd1 = c1;
            const bool in_ok = ND == 1 || (si0 >= 0 && si0 < dims0 && (ND < 3 || (si1 >= 0 && si1 < d1)));
            const bool dy_ok = ND == 1 || (sd0 < dims0 && (ND < 3 || sd1 < d1));
            const long long rbase_in = ND == 1 ? 0 : (ND == 2 ? (long long)si0 * d1 : ((long long)si0 * d1 + si1) * d2);
            const long long rbase_dy = ND == 1 ? 0 : (ND == 2 ? (long long)sd0 * d1 : ((long long)sd0 * d1 + sd1) * d2);
            for (int e = wl; e < pdl * CG; e += 32) {
                const int px = e / CG, l = e - px * CG;
                const int slot = cf_slot(row * pdl + px) * CG + l;
                // innermost source coordinate (for 1D the innermost axis is axis 0, offset by the slab)
                const int xi = (ND == 1 ? z0 : 0) + px - H, xd = (ND == 1 ? z0 : 0) + px;
                if (FWD || BWD) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (in_ok && xi >= 0 && xi < dl_) v = in[(ibase + rbase_in + xi) * D4 + lane0 + l];
                    sIN[slot] = v;
                }
                if (BWD) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (dy_ok && xd < dl_) v = dy[(ibase + rbase_dy + xd) * D4 + lane0 + l];
                    sDY[slot] = v;
                }
            }
        }
    }
    __syncthreads();

    // ---- compute: work item = (run of R points along the innermost axis, N channels)
    const int lane = tid % NL;
    const int ch = lane0 * 4 + lane * N;                     // first channel of this thread
    const float* sINf = (const float*)sIN;
    const float* sDYf = (const float*)sDY;
    const int lo = lane * N;                                 // float offset inside a point's 4 CG channels
    auto ldin = [&](int pt) { return *(const V*)(sINf + cf_slot(pt) * (CG * 4) + lo); };
    auto lddy = [&](int pt) { return *(const V*)(sDYf + cf_slot(pt) * (CG * 4) + lo); };
    V kv[T::V];
#pragma unroll
    for (int k = 0; k < T::V; k++) kv[k] = *(const V*)(ker + (long long)k * c.D + ch);
    const V b0 = (FWD && bias) ? *(const V*)(bias + ch) : cf_zero<V>();
    V dk[BWD ? T::V + 1 : 1];
#pragma unroll
    for (int k = 0; k < (BWD ? T::V + 1 : 1); k++) dk[k] = cf_zero<V>();
    const int dlast = ND == 1 ? dims0 : (ND == 2 ? d1 : d2);   // innermost extent
    const int nrun_line = dlast / R;
    const int lines = ND == 1 ? 1 : (ND == 2 ? nz : nz * d1);
    const int nwork = (ND == 1 ? (nz / R) : lines * nrun_line);
    for (int wi = tid / NL; wi < nwork; wi += CF_THREADS / NL) {
        // coordinates of the run's first point (relative to the slab for axis 0)
        int zr, y = 0, x0;
        if (ND == 1) {
            zr = wi * R;
            x0 = zr;
        } else if (ND == 2) {
            zr = wi / nrun_line;
            x0 = (wi - zr * nrun_line) * R;
        } else {
            const int ln = wi / nrun_line;
            zr = ln / d1;
            y = ln - zr * d1;
            x0 = (wi - ln * nrun_line) * R;
        }
        // padded base index of the run (the same expression for the input, whose halo is on the low
        // side of every axis, and for dy, whose halo is on the high side)
        int base;
        if (ND == 1) base = zr;
        else if (ND == 2) base = zr * g.ps[0] + x0;
        else base = zr * g.ps[0] + y * g.ps[1] + x0;
        V acc[R], adin[R], dyo[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            acc[r] = b0;
            adin[r] = cf_zero<V>();
        }
        if (BWD) {
#pragma unroll
            for (int r = 0; r < R; r++) dyo[r] = lddy(base + r);
        }
#pragma unroll
        for (int row = 0; row < T::ROWS; row++) {
            // outer digits of this row: (k0) for 2D, (k0, k1) for 3D; shift of an axis = H - digit
            const int k0 = ND == 3 ? row / K : row;
            const int k1 = ND == 3 ? row % K : 0;
            int rin, rdy;
            if (ND == 1) {
                rin = base;
                rdy = base;
            } else if (ND == 2) {
                rin = base + k0 * g.ps[0];
                rdy = base + (H - k0) * g.ps[0];
            } else {
                rin = base + k0 * g.ps[0] + k1 * g.ps[1];
                rdy = base + (H - k0) * g.ps[0] + (H - k1) * g.ps[1];
            }
            {
                V w[R + H];
#pragma unroll
                for (int j = 0; j < R + H; j++) w[j] = ldin(rin + j);
#pragma unroll
                for (int kx = 0; kx < K; kx++) {
                    const int k = row * K + kx;
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        // in[x - (H - kx)] with x = x0 + r sits at padded x0 + r + kx
                        if (FWD) cf_fma(acc[r], w[r + kx], kv[k]);
                        if (BWD) cf_fma(dk[k], dyo[r], w[r + kx]);
                    }
                }
            }
            if (BWD) {
                V w[R + H];
#pragma unroll
                for (int j = 0; j < R + H; j++) w[j] = lddy(rdy + j);
#pragma unroll
                for (int kx = 0; kx < K; kx++) {
                    const int k = row * K + kx;
#pragma unroll
                    for (int r = 0; r < R; r++) cf_fma(adin[r], w[r + H - kx], kv[k]);   // dy[x + (H - kx)]
                }
            }
        }
        // global point index of the run's first point
        long long p;
        if (ND == 1) p = z0 + zr;
        else if (ND == 2) p = (long long)(z0 + zr) * d1 + x0;
        else p = ((long long)(z0 + zr) * d1 + y) * d2 + x0;
#pragma unroll
        for (int r = 0; r < R; r++) {
            const long long gi = (ibase + p + r) * c.D + ch;
            if (FWD) *(V*)(out + gi) = acc[r];
            if (BWD) {
                *(V*)(din + gi) = adin[r];
                cf_add(dk[T::V], dyo[r]);
            }
        }
    }
    if (!BWD) return;
    // ---- dkernel / dbias partials of the CTA, a fixed-order tree: the threads of a warp that share a
    // channel lane (xor shuffles over the lane-stride offsets), then the warps in order
    constexpr int NV = T::V + 1;
#pragma unroll
    for (int k = 0; k < NV; k++)
#pragma unroll
        for (int o = NL; o < 32; o <<= 1) cf_add(dk[k], cf_shfl(dk[k], o));
    __syncthreads();
    V* red = (V*)cf_smem;   // reuse the staging area: [warp][NV][NL]
    if (wl < NL) {
#pragma unroll
        for (int k = 0; k < NV; k++) red[(warp * NV + k) * NL + wl] = dk[k];
    }
    __syncthreads();
    const long long chunk = b * g.nslab + slab;
    for (int i = tid; i < NV * NL; i += CF_THREADS) {
        const int k = i / NL, l = i - k * NL;
        V s2 = red[k * NL + l];
        for (int wv = 1; wv < CF_THREADS / 32; wv++) cf_add(s2, red[(wv * NV + k) * NL + l]);
        *(V*)(part + (chunk * NV + k) * c.D + lane0 * 4 + l * N) = s2;
    }
}

// ---------------------------------------------------------------------------
// 3D variant (K = 2 or 3, D a multiple of 4), streaming along axis 0.  A CTA
// owns (item, slab of T0 planes of axis 0, 4 channels) and walks its output
// planes in order.  Planes are staged with cp.async (16 bytes = 4 channels per
// point, zero-filled outside the grid) into a ring of NS plane slots per
// tensor: stage s holds the input plane z0 - H + s and the dy plane z0 + s,
// each laid out as [row][PX] points with PX = d2 + K - 1 rounded up to an odd
// number.  Output plane zr uses stages zr .. zr + H; stage zr + NS - 1 is
// issued at the top of iteration zr, into the slot that output zr - 1 freed,
// so the copies of the next planes overlap the arithmetic of this one, and
// every input and dy plane is read once per slab.
// Per plane, a warp takes 8 consecutive rows (axis 1) at one run of R points
// along axis 2, 4 threads per point (one channel each): the 8 rows of a warp
// sit PX points apart, and with PX odd their 16-byte points fall in 8
// different bank groups, so every shared-memory read is conflict-free and its
// address is the thread's run base plus a per-row constant.  Arithmetic per
// point and its order are those of the generic fused kernel.
// ---------------------------------------------------------------------------
constexpr int CF3_NS = 8;   // plane slots per tensor

struct Fused3Geom {
    int T0, nslab;   // planes of axis 0 per slab, slabs per item
    int PX, PY;      // padded row pitch (odd) and rows per plane, in points
    int slot;        // floats of one plane slot (128-byte multiple)
};

__device__ __forceinline__ void cf_cp16(uint32_t sdst, const void* gsrc, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sdst), "l"(gsrc), "r"(ok ? 16 : 0)
                 : "memory");
}

template <int K, int R, int MODE>
__global__ void __launch_bounds__(CF_THREADS, 2) conv_fused3d_kernel(ConvDesc c, Fused3Geom g,
                                                                     const float4* __restrict__ in,
                                                                     const float* __restrict__ ker,
                                                                     const float* __restrict__ bias,
                                                                     const float4* __restrict__ dy,
                                                                     float* __restrict__ out,
                                                                     float* __restrict__ din,
                                                                     float* __restrict__ part) {
    constexpr int H = K - 1, V = K * K * K, ROWS = K * K, NS = CF3_NS;
    constexpr bool FWD = MODE & 1, BWD = (MODE & 2) != 0;
    extern __shared__ __align__(128) float cf3_smem[];
    float* sIN = cf3_smem;                                   // [NS][slot]
    float* sDY = cf3_smem + NS * g.slot;
    const int slab = blockIdx.x % g.nslab;
    const int b = blockIdx.x / g.nslab;
    const int q = blockIdx.y;                                // float4 channel lane of this CTA
    const int d0 = (int)c.dims[0], d1 = (int)c.dims[1], d2 = (int)c.dims[2];
    const int z0 = slab * g.T0;
    const int nz = min(g.T0, d0 - z0);
    const int nstage = nz + H;
    const int D4 = c.D >> 2;
    const int tid = threadIdx.x, wl = tid & 31, warp = tid >> 5;
    const int pdx = d2 + H, npt = (d1 + H) * pdx;            // staged points of one padded plane
    const long long zstride = (long long)d1 * d2 * D4;       // float4s per plane of axis 0
    const float4* inb = in + (long long)b * c.P * D4 + q;
    const float4* dyb = BWD ? dy + (long long)b * c.P * D4 + q : inb;
    const uint32_t uin = smem_u32(sIN), udy = smem_u32(sDY);

    // stage st -> slot st % NS: padded (py, px) <- input (z0 - H + st, py - H, px - H), dy (z0 + st, py, px)
    auto stage = [&](int st) {
        if (st < nstage) {
            const int sl = st % NS;
            const int zi = z0 - H + st, zd = z0 + st;
            const bool zi_ok = zi >= 0, zd_ok = zd < d0;
            int py = tid / pdx, px = tid - py * pdx;
            const int sy = CF_THREADS / pdx, sx = CF_THREADS - sy * pdx;
            for (int i = tid; i < npt; i += CF_THREADS) {
                const uint32_t so = (uint32_t)((sl * g.slot + (py * g.PX + px) * 4) * 4);
                {
                    const int yi = py - H, xi = px - H;
                    const bool ok = zi_ok && yi >= 0 && xi >= 0;
                    cf_cp16(uin + so, ok ? inb + zi * zstride + ((long long)yi * d2 + xi) * D4 : inb, ok);
                }
                if (BWD) {
                    const bool ok = zd_ok && py < d1 && px < d2;
                    cf_cp16(udy + so, ok ? dyb + zd * zstride + ((long long)py * d2 + px) * D4 : dyb, ok);
                }
                px += sx;
                py += sy;
                if (px >= pdx) {
                    px -= pdx;
                    py++;
                }
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    for (int st = 0; st < NS - 1; st++) stage(st);

    const int l = tid & 3, iy = (tid >> 2) & 7;
    const int ch = q * 4 + l;
    float kv[V];
#pragma unroll
    for (int k = 0; k < V; k++) kv[k] = ker[(long long)k * c.D + ch];
    const float b0 = (FWD && bias) ? bias[ch] : 0.0f;
    float dk[BWD ? V + 1 : 1];
#pragma unroll
    for (int k = 0; k < (BWD ? V + 1 : 1); k++) dk[k] = 0.0f;
    const int PX = g.PX;
    const int nrun = d2 / R, nyb = (d1 + 7) >> 3;
    const int ntask = nyb * nrun;
    const long long ibase = (long long)b * c.P;
    for (int zr = 0; zr < nz; zr++) {
        // stages <= zr + H have landed once at most NS - 2 - H of the later groups are pending
        asm volatile("cp.async.wait_group %0;\n" ::"n"(NS - 2 - H) : "memory");
        __syncthreads();   // ... for every thread's copies; and every warp is done with output zr - 1
        stage(zr + NS - 1);   // into the slot of stage zr - 1
        const float* pin[K];
        const float* pdy[K];
#pragma unroll
        for (int k0 = 0; k0 < K; k0++) {
            pin[k0] = sIN + ((zr + k0) % NS) * g.slot + l;              // input plane z - H + k0
            pdy[k0] = sDY + ((zr + H - k0) % NS) * g.slot + l;          // dy plane z + H - k0
        }
        for (int t = warp; t < ntask; t += CF_THREADS / 32) {
            const int yb = t / nrun;
            const int y = yb * 8 + iy;
            if (y >= d1) continue;
            const int x0 = (t - yb * nrun) * R;
            const int base = (y * PX + x0) * 4;
            float acc[R], adin[R], dyo[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
                acc[r] = b0;
                adin[r] = 0.0f;
                if (BWD) dyo[r] = pdy[H][base + r * 4];
            }
#pragma unroll
            for (int row = 0; row < ROWS; row++) {
                const int k0 = row / K, k1 = row % K;
                {
                    const float* pr = pin[k0] + base + k1 * PX * 4;
                    float w[R + H];
#pragma unroll
                    for (int j = 0; j < R + H; j++) w[j] = pr[j * 4];
#pragma unroll
                    for (int kx = 0; kx < K; kx++) {
                        const int k = row * K + kx;
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            if (FWD) acc[r] = __fmaf_rn(w[r + kx], kv[k], acc[r]);
                            if (BWD) dk[k] = __fmaf_rn(dyo[r], w[r + kx], dk[k]);
                        }
                    }
                }
                if (BWD) {
                    const float* pr = pdy[k0] + base + (H - k1) * PX * 4;
                    float w[R + H];
#pragma unroll
                    for (int j = 0; j < R + H; j++) w[j] = pr[j * 4];
#pragma unroll
                    for (int kx = 0; kx < K; kx++) {
                        const int k = row * K + kx;
#pragma unroll
                        for (int r = 0; r < R; r++) adin[r] = __fmaf_rn(w[r + H - kx], kv[k], adin[r]);
                    }
                }
            }
            const long long gi0 = (ibase + ((long long)(z0 + zr) * d1 + y) * d2 + x0) * c.D + ch;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (FWD) out[gi0 + (long long)r * c.D] = acc[r];
                if (BWD) {
                    din[gi0 + (long long)r * c.D] = adin[r];
                    dk[V] += dyo[r];
                }
            }
        }
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    if (!BWD) return;
    // ---- dkernel / dbias partials of the CTA: the 8 threads of a warp that share a channel
    // (xor shuffles 4, 8, 16), then the warps in order
    constexpr int NV = V + 1;
#pragma unroll
    for (int k = 0; k < NV; k++)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) dk[k] += __shfl_xor_sync(~0u, dk[k], o);
    __syncthreads();   // every warp is done with the ring
    float* red = cf3_smem;   // [warp][NV][4]
    if (wl < 4) {
#pragma unroll
        for (int k = 0; k < NV; k++) red[(warp * NV + k) * 4 + wl] = dk[k];
    }
    __syncthreads();
    const long long chunk = (long long)b * g.nslab + slab;
    for (int i = tid; i < NV * 4; i += CF_THREADS) {
        const int k = i >> 2, l2 = i & 3;
        float s2 = red[k * 4 + l2];
        for (int wv = 1; wv < CF_THREADS / 32; wv++) s2 += red[(wv * NV + k) * 4 + l2];
        part[(chunk * NV + k) * c.D + q * 4 + l2] = s2;
    }
}

static bool cf3_plan(const ConvDesc& c, int mode, Fused3Geom* g, int* smem, int* R) {
    if (c.nd != 3 || c.K < 2 || c.K > 3 || c.D % 4 != 0) return false;
    const int H = c.K - 1;
    const long long d0 = c.dims[0], d1 = c.dims[1], d2 = c.dims[2];
    if (d1 + H > 4096 || d2 + H > 4096 || c.batch > 0x7fffffffLL) return false;
    int PX = (int)d2 + H;
    if (PX % 2 == 0) PX++;
    const int PY = (int)d1 + H;
    const int ntens = (mode & 2) ? 2 : 1;
    const long long slot = ((long long)PX * PY * 16 + 127) / 128 * 128;
    if (CF3_NS * slot * ntens > CF_SMEM_MAX) return false;
    // slabs along axis 0: enough CTAs for about six waves at two per SM, at least 4 planes per slab
    long long nslab = 1;
    const long long per_slab = c.batch * (c.D / 4);
    while (nslab < d0 / 4 && per_slab * nslab < 6 * 148 * 2) nslab++;
    g->nslab = (int)nslab;
    g->T0 = (int)((d0 + nslab - 1) / nslab);
    g->nslab = (int)((d0 + g->T0 - 1) / g->T0);
    g->PX = PX;
    g->PY = PY;
    g->slot = (int)(slot / 4);
    *R = (d2 % 4 == 0) ? 4 : 1;
    int sm = (int)(CF3_NS * slot * ntens);
    const int red = (CF_THREADS / 32) * (c.K * c.K * c.K + 1) * 4 * 4;
    if ((mode & 2) && red > sm) sm = red;
    *smem = sm;
    return true;
}

template <int K, int R, int MODE>
static cudaError_t cf3_launch_t(const ConvDesc& c, const Fused3Geom& g, int smem, const float* in, const float* ker,
                                const float* bias, const float* dy, float* out, float* din, float* part,
                                cudaStream_t st) {
    auto k = conv_fused3d_kernel<K, R, MODE>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    dim3 grid((unsigned)(c.batch * g.nslab), (unsigned)(c.D / 4));
    k<<<grid, CF_THREADS, smem, st>>>(c, g, (const float4*)in, ker, bias, (const float4*)dy, out, din, part);
    return cudaGetLastError();
}

template <int K, int R>
static cudaError_t cf3_mode(int mode, const ConvDesc& c, const Fused3Geom& g, int smem, const float* in,
                            const float* ker, const float* bias, const float* dy, float* out, float* din,
                            float* part, cudaStream_t st) {
    switch (mode) {
        case 1: return cf3_launch_t<K, R, 1>(c, g, smem, in, ker, bias, dy, out, din, part, st);
        case 2: return cf3_launch_t<K, R, 2>(c, g, smem, in, ker, bias, dy, out, din, part, st);
        default: return cf3_launch_t<K, R, 3>(c, g, smem, in, ker, bias, dy, out, din, part, st);
    }
}

// dkernel[i] (i < V D) and dbias[i - V D] = sum over the chunks of part[chunk][i], fixed order (one launch)
__global__ void cf_reduce_dk(const float* __restrict__ part, float* __restrict__ dker, float* __restrict__ dbias,
                             long long VD, int D, long long nch) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = VD + D;
    if (i >= (dbias ? stride : VD)) return;
    float acc = 0.0f;
    for (long long j = 0; j < nch; j++) acc += part[j * stride + i];
    if (i < VD) dker[i] = acc;
    else dbias[i - VD] = acc;
}

// Channel lanes per CTA: 8 channels (one 32-byte sector per point).
static int cf_cg(int) { return 2; }

// Plans the slab split; false when the shape is outside the kernel's set.
static bool cf_plan(const ConvDesc& c, int mode, FusedGeom* g, int* smem, int* R) {
    if (c.nd < 1 || c.nd > 2 || c.K < 2 || c.K > 4 || c.D % 8 != 0) return false;
    const int H = c.K - 1, CG = cf_cg(c.nd);
    const int dlast = (int)c.dims[c.nd - 1];
    *R = (dlast % 4 == 0) ? 4 : 1;
    int rest = 1;   // padded points of one plane of axis 0
    for (int a = 1; a < c.nd; a++) rest *= (int)c.dims[a] + H;
    const int ntens = (mode & 2) ? 2 : 1;
    auto bytes = [&](int T0) {
        const int pts = (T0 + H) * rest;
        return (pts + pts / 4 + 1) * CG * 16 * ntens;
    };
    int T0 = (int)c.dims[0];
    if (c.nd == 1) {
        T0 = (int)c.dims[0] < 1024 ? (int)c.dims[0] : 1024;
        T0 = T0 / *R * *R;
        if (T0 < *R) T0 = *R;
    }
    const int smax = CF_SMEM_MAX;
    while (T0 > 1 && bytes(T0) > smax) T0 = c.nd == 1 ? T0 / 2 / *R * *R : T0 - 1;
    if (T0 < 1 || bytes(T0) > smax) return false;
    if (c.nd == 1 && T0 % *R) return false;
    g->T0 = T0;
    g->nslab = (int)((c.dims[0] + T0 - 1) / T0);
    if (c.nd == 1 && c.dims[0] % T0 != 0 && (c.dims[0] % T0) % *R != 0) return false;
    g->pd[0] = T0 + H;
    for (int a = 1; a < c.nd; a++) g->pd[a] = (int)c.dims[a] + H;
    for (int a = c.nd; a < 3; a++) g->pd[a] = 1;
    g->ps[c.nd - 1] = 1;
    for (int a = c.nd - 2; a >= 0; a--) g->ps[a] = g->ps[a + 1] * g->pd[a + 1];
    g->slab_pts = g->pd[0] * g->ps[0];
    g->slab_slots = g->slab_pts + g->slab_pts / 4 + 1;
    int sm = bytes(T0);
    const int vol = (int)(std::pow((double)c.K, (double)c.nd) + 0.5) + 1;
    const int red = (CF_THREADS / 32) * vol * 16 * 4;   // [warp][V + 1][lanes] partials, at most 16 B x 4 lanes
    if ((mode & 2) && red > sm) sm = red;
    *smem = sm;
    return true;
}

long long conv_fused_chunks(const ConvDesc& c, int mode) {
    int sm, R;
    if (c.nd == 3) {
        Fused3Geom g3;
        if (!cf3_plan(c, mode, &g3, &sm, &R)) return -1;
        return c.batch * g3.nslab;
    }
    FusedGeom g;
    if (!cf_plan(c, mode, &g, &sm, &R)) return -1;
    return c.batch * g.nslab;
}

template <int ND, int K, int R, int MODE>
static cudaError_t cf_launch_t(const ConvDesc& c, const FusedGeom& g, int smem, const float* in, const float* ker,
                               const float* bias, const float* dy, float* out, float* din, float* part,
                               cudaStream_t st) {
    // two channels per thread as packed fp32 pairs, 8 channels per CTA (1D and 2D; 3D has its own kernel)
    constexpr int N = 2;
    constexpr int CG = 2;
    auto k = conv_fused_kernel<ND, K, R, MODE, N, CG>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    dim3 grid((unsigned)(c.batch * g.nslab), (unsigned)(c.D / 4 / CG));
    k<<<grid, CF_THREADS, smem, st>>>(c, g, (const float4*)in, ker, bias, (const float4*)dy, out, din, part);
    return cudaGetLastError();
}

template <int ND, int K, int R>
static cudaError_t cf_mode(int mode, const ConvDesc& c, const FusedGeom& g, int smem, const float* in,
                           const float* ker, const float* bias, const float* dy, float* out, float* din, float* part,
                           cudaStream_t st) {
    switch (mode) {
        case 1: return cf_launch_t<ND, K, R, 1>(c, g, smem, in, ker, bias, dy, out, din, part, st);
        case 2: return cf_launch_t<ND, K, R, 2>(c, g, smem, in, ker, bias, dy, out, din, part, st);
        default: return cf_launch_t<ND, K, R, 3>(c, g, smem, in, ker, bias, dy, out, din, part, st);
    }
}

// mode 1: forward; 2: backward; 3: both.  part: >= conv_fused_chunks * (V + 1) * D floats (backward).
// cudaErrorNotSupported outside the kernel's set or when nch_max is too small.
cudaError_t launch_conv_fused(const ConvDesc& c, int mode, const float* in, const float* ker, const float* bias,
                              float* out, const float* dy, float* din, float* dker, float* dbias, float* part,
                              long long nch_max, cudaStream_t st) {
    FusedGeom g;
    Fused3Geom g3;
    int smem, R;
    if (c.nd == 3) {
        if (!cf3_plan(c, mode, &g3, &smem, &R)) return cudaErrorNotSupported;
        g.nslab = g3.nslab;
    } else if (!cf_plan(c, mode, &g, &smem, &R)) {
        return cudaErrorNotSupported;
    }
    const long long nch = c.batch * g.nslab;
    if ((mode & 2) && nch > nch_max) return cudaErrorNotSupported;
    if (c.batch * g.nslab > 0x7fffffffLL) return cudaErrorNotSupported;
    const uintptr_t al = (uintptr_t)in | (uintptr_t)ker | (uintptr_t)(bias ? bias : ker) |
                         (uintptr_t)(out ? out : ker) | (uintptr_t)(dy ? dy : ker) | (uintptr_t)(din ? din : ker) |
                         (uintptr_t)(part ? part : ker);
    if (al & 15) return cudaErrorNotSupported;
    cudaError_t e;
#define KMB_CF(ND_, K_)                                                                                        \
    if (c.nd == ND_ && c.K == K_)                                                                              \
        e = R == 4 ? cf_mode<ND_, K_, 4>(mode, c, g, smem, in, ker, bias, dy, out, din, part, st)              \
                   : cf_mode<ND_, K_, 1>(mode, c, g, smem, in, ker, bias, dy, out, din, part, st);             \
    else
    // 3D: the conflict-free variant (K = 4 is left to the other kernels: 64 dkernel accumulators
    // per thread do not fit)
    if (c.nd == 3 && c.K == 2)
        e = R == 4 ? cf3_mode<2, 4>(mode, c, g3, smem, in, ker, bias, dy, out, din, part, st)
                   : cf3_mode<2, 1>(mode, c, g3, smem, in, ker, bias, dy, out, din, part, st);
    else if (c.nd == 3 && c.K == 3)
        e = R == 4 ? cf3_mode<3, 4>(mode, c, g3, smem, in, ker, bias, dy, out, din, part, st)
                   : cf3_mode<3, 1>(mode, c, g3, smem, in, ker, bias, dy, out, din, part, st);
    else
    KMB_CF(1, 2) KMB_CF(1, 3) KMB_CF(1, 4) KMB_CF(2, 2) KMB_CF(2, 3) KMB_CF(2, 4)
    return cudaErrorNotSupported;
#undef KMB_CF
    if (e != cudaSuccess || !(mode & 2)) return e;
    const long long V = (long long)(std::pow((double)c.K, (double)c.nd) + 0.5);
    const long long cnt = (V + 1) * c.D;
    cf_reduce_dk<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(part, dker, dbias, V * c.D, c.D, nch);
    return cudaGetLastError();
}

}  // namespace kmb
