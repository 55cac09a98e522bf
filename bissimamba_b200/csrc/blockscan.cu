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
#include "../../include/kmamba_block.h"

namespace kmb {

constexpr int BS_MAXND = 8;

__device__ __forceinline__ float ldv(const float* p) { return *p; }
__device__ __forceinline__ float ldv(const __nv_bfloat16* p) { return __bfloat162float(*p); }

struct BSDesc {
    int nd, N, R, P2, fast, bf16;
    float deflam;
    long long L, batch;
    int dims[BS_MAXND], strides[BS_MAXND];
    int nlev;
    const int* lev_start;   // [nlev + 1]
    const int* lev_pts;     // [L]
    const void *u, *dt, *lam, *B, *C;  // float, or __nv_bfloat16 when bf16
    const float *A, *theta;
    float *h, *Bu, *y;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void bs_unravel(const BSDesc& s, int t, int* idx) {
    for (int k = 0; k < s.nd; k++) idx[k] = (t / s.strides[k]) % s.dims[k];
}

template <typename T>
__global__ void __launch_bounds__(512) blockscan_fwd_kernel(BSDesc s) {
    const int b = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R;
    const int n0 = 2 * lane, n1 = 2 * lane + 1;
    const bool h0ok = n0 < N, h1ok = n1 < N, pair = h1ok;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        cth = cosf(s.theta[lane]);
        sth = sinf(s.theta[lane]);
    }
    const long long L = s.L;
    const T* u = (const T*)s.u + b * L * R;
    const T* dtp = (const T*)s.dt + b * L;
    const T* lamp = s.lam ? (const T*)s.lam + b * L : nullptr;
    const T* Bp = (const T*)s.B + b * L * NR;
    const T* Cp = (const T*)s.C + b * L * NR;
    float* h = s.h + b * L * N;
    float* Bu = s.Bu + b * L * N;
    float* y = s.y + b * L * R;
    for (int lev = 0; lev < s.nlev; lev++) {
        const int beg = s.lev_start[lev], end = s.lev_start[lev + 1];
        for (int i = beg + warp; i < end; i += nw) {
            const int t = s.lev_pts[i];
            const float dt = ldv(dtp + t);
            const float lam = lamp ? ldv(lamp + t) : s.deflam;
            float bu0 = 0.0f, bu1 = 0.0f;
            for (int r = 0; r < R; r++) {
                const float ur = ldv(u + (long long)t * R + r);
                if (h0ok) bu0 = __fmaf_rn(ldv(Bp + (long long)t * NR + r * N + n0), ur, bu0);
                if (h1ok) bu1 = __fmaf_rn(ldv(Bp + (long long)t * NR + r * N + n1), ur, bu1);
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
                    const long long q = (long long)(t - s.strides[k]) * N;
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
                const float g = lam * dt;
                hn0 = __fmaf_rn(g, bu0, hn0);
                hn1 = __fmaf_rn(g, bu1, hn1);
            } else {
                // 1D recurrence (reference src/mamba_block.c:384-393)
                float p0 = 0.0f, p1 = 0.0f, pb0 = 0.0f, pb1 = 0.0f;
                if (t > 0) {
                    const long long q = (long long)(t - 1) * N;
                    if (h0ok) { p0 = h[q + n0]; pb0 = Bu[q + n0]; }
                    if (h1ok) { p1 = h[q + n1]; pb1 = Bu[q + n1]; }
                }
                const float r0 = pair ? cth * p0 - sth * p1 : p0;
                const float r1 = sth * p0 + cth * p1;
                const float beta0 = (1.0f - lam) * dt * al0, beta1 = (1.0f - lam) * dt * al1;
                const float g = lam * dt;
                hn0 = __fmaf_rn(g, bu0, __fmaf_rn(beta0, pb0, al0 * r0));
                hn1 = __fmaf_rn(g, bu1, __fmaf_rn(beta1, pb1, al1 * r1));
            }
            const long long o = (long long)t * N;
            if (h0ok) { h[o + n0] = hn0; Bu[o + n0] = bu0; }
            if (h1ok) { h[o + n1] = hn1; Bu[o + n1] = bu1; }
            for (int r = 0; r < R; r++) {
                float part = 0.0f;
                if (h0ok) part = ldv(Cp + (long long)t * NR + r * N + n0) * hn0;
                if (h1ok) part = __fmaf_rn(ldv(Cp + (long long)t * NR + r * N + n1), hn1, part);
                part = warp_sum(part);
                if (lane == 0) y[(long long)t * R + r] = part;
            }
        }
        __syncthreads();
    }
}

struct BSGrad {
    const float* dy;
    float *dB, *dC, *du, *ddt, *dlam;
    float* G;     // scratch [batch, L, N]
    float* pA;    // scratch [batch, N]
    float* pth;   // scratch [batch, 32]
};

template <typename T>
__global__ void __launch_bounds__(512) blockscan_bwd_kernel(BSDesc s, BSGrad g) {
    const int b = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int N = s.N, R = s.R, NR = N * R, nd = s.nd < 1 ? 1 : s.nd;
    const int n0 = 2 * lane, n1 = 2 * lane + 1;
    const bool h0ok = n0 < N, h1ok = n1 < N, pair = h1ok;
    const float A0 = h0ok ? s.A[n0] : 0.0f, A1 = h1ok ? s.A[n1] : 0.0f;
    float cth = 1.0f, sth = 0.0f;
    if (pair) {
        cth = cosf(s.theta[lane]);
        sth = sinf(s.theta[lane]);
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
        for (int i = beg + warp; i < end; i += nw) {
            const int t = s.lev_pts[i];
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
                const float G0 = h0ok ? G[(long long)sp * N + n0] : 0.0f;
                const float G1 = h1ok ? G[(long long)sp * N + n1] : 0.0f;
                a0 += al0 * G0;
                a1 += al1 * G1;
                ab0 += coef * al0 * G0;
                ab1 += coef * al1 * G1;
            }
            float gh0 = pair ? cth * a0 + sth * a1 : a0;
            float gh1 = -sth * a0 + cth * a1;
            const long long o = (long long)t * N;
            const float ht0 = h0ok ? h[o + n0] : 0.0f, ht1 = h1ok ? h[o + n1] : 0.0f;
            if (pair) {
                const float hat0 = cth * ht0 - sth * ht1, hat1 = sth * ht0 + cth * ht1;
                gth += -a0 * hat1 + a1 * hat0;
            }
            for (int r = 0; r < R; r++) {
                const float dyr = dy[(long long)t * R + r];
                const long long c0 = (long long)t * NR + r * N;
                if (h0ok) {
                    gh0 += ldv(Cp + c0 + n0) * dyr;
                    g.dC[b * L * NR + c0 + n0] += dyr * ht0;
                }
                if (h1ok) {
                    gh1 += ldv(Cp + c0 + n1) * dyr;
                    g.dC[b * L * NR + c0 + n1] += dyr * ht1;
                }
            }
            if (h0ok) G[o + n0] = gh0;
            if (h1ok) G[o + n1] = gh1;
            const float bu0 = h0ok ? Bu[o + n0] : 0.0f, bu1 = h1ok ? Bu[o + n1] : 0.0f;
            const float gam = lam * dt;
            const float gbu0 = gam * gh0 + ab0, gbu1 = gam * gh1 + ab1;
            for (int r = 0; r < R; r++) {
                const float ur = ldv(u + (long long)t * R + r);
                const long long c0 = (long long)t * NR + r * N;
                float part = 0.0f;
                if (h0ok) {
                    g.dB[b * L * NR + c0 + n0] += gbu0 * ur;
                    part += gbu0 * ldv(Bp + c0 + n0);
                }
                if (h1ok) {
                    g.dB[b * L * NR + c0 + n1] += gbu1 * ur;
                    part += gbu1 * ldv(Bp + c0 + n1);
                }
                part = warp_sum(part);
                if (lane == 0) g.du[b * L * R + (long long)t * R + r] += part;
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
                gA0 += dz0 * dt;
                gA1 += dz1 * dt;
                const float ds = al0 * sb0 * gh0 + al1 * sb1 * gh1;
                gdt += (1.0f - lam) * inv * ds;
                glam -= dt * inv * ds;
            }
            gdt = warp_sum(gdt);
            glam = warp_sum(glam);
            if (lane == 0) {
                if (g.ddt) g.ddt[b * L + t] += gdt;
                if (g.dlam) g.dlam[b * L + t] += glam;
            }
        }
        __syncthreads();
    }
    // per-item partials: sum the warps' accumulators in a fixed order
    __shared__ float sA[16][64];
    __shared__ float sT[16][32];
    sA[warp][n0 & 63] = gA0;
    sA[warp][n1 & 63] = gA1;
    sT[warp][lane] = gth;
    __syncthreads();
    if (warp == 0) {
        float t0 = 0.0f, t1 = 0.0f, tt = 0.0f;
        for (int w = 0; w < nw; w++) {
            t0 += sA[w][n0 & 63];
            t1 += sA[w][n1 & 63];
            tt += sT[w][lane];
        }
        if (h0ok) g.pA[(long long)b * N + n0] = t0;
        if (h1ok) g.pA[(long long)b * N + n1] = t1;
        g.pth[(long long)b * 32 + lane] = tt;
    }
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
#include <cstring>
#include <map>
#include <vector>
#include "../../include/wavefront_plan.h"

namespace kmb {
void* workspace(int slot, size_t bytes);
int set_error(const char* msg);
int set_cuda_error(const char* where, cudaError_t e);
enum { WS_BS_SCRATCH = 4 };

// Device copy of the wavefront plan of `dims` (level starts [nlev + 1], then the
// points of every level [L]), cached per host thread, device and shape.
// Shared with the Scan-A backward (scannd_bwd.cu).
struct PlanEntry {
    int nlev = 0;
    int* dev = nullptr;
};
static thread_local std::map<int, std::map<std::vector<long>, PlanEntry>> tl_plans;

int device_plan(const std::vector<long>& dims, long L, int** out, int* nlev, cudaStream_t st) {
    int devid = 0;
    cudaGetDevice(&devid);
    PlanEntry& pe = tl_plans[devid][dims];
    if (pe.dev) {
        *out = pe.dev;
        *nlev = pe.nlev;
        return 0;
    }
    KMWavefrontPlan* pl = km_wavefront_plan_create(dims.data(), (long)dims.size(), 0);
    if (!pl) return set_error("cannot build the wavefront plan");
    const int nl = (int)pl->max_level + 1;
    std::vector<int> host(nl + 1 + L);
    for (int i = 0; i <= nl; i++) host[i] = (int)pl->level_starts[i];
    for (long i = 0; i < L; i++) host[nl + 1 + i] = (int)pl->level_offsets[i];
    km_wavefront_plan_free(pl);
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
    *out = d;
    *nlev = nl;
    return 0;
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
    if (p->L > 0x7fffffffL) return set_error("blockscan: L too large");
    memset(s, 0, sizeof(*s));
    s->nd = p->ndims <= 1 ? 1 : (int)p->ndims;
    s->N = (int)p->N;
    s->R = (int)p->R;
    s->P2 = (s->N + 1) / 2;
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
    if (device_plan(dims, p->L, &plan, &s->nlev, st)) return -1;
    s->lev_start = plan;
    s->lev_pts = plan + s->nlev + 1;
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

}  // namespace kmb

using namespace kmb;

extern "C" int kmb_blockscan_forward(const KMBlockScanParams* p, long batch, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    BSDesc s;
    if (bs_desc(p, batch, &s, st)) return -1;
    if (s.bf16) blockscan_fwd_kernel<__nv_bfloat16><<<(unsigned)batch, bs_threads(s), 0, st>>>(s);
    else blockscan_fwd_kernel<float><<<(unsigned)batch, bs_threads(s), 0, st>>>(s);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("blockscan_fwd", e);
}

extern "C" int kmb_blockscan_backward(const KMBlockScanParams* p, long batch, const float* dy,
                                      const KMBlockScanGrads* gr, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (!dy || !gr || !gr->dB || !gr->dC || !gr->du) return set_error("blockscan backward: dy, dB, dC, du required");
    BSDesc s;
    if (bs_desc(p, batch, &s, st)) return -1;
    const size_t nG = (size_t)batch * s.L * s.N;
    const size_t bytes = (nG + (size_t)batch * s.N + (size_t)batch * 32) * sizeof(float) + 512;
    char* w = (char*)workspace(WS_BS_SCRATCH, bytes);
    if (!w) return set_error("workspace allocation failed");
    BSGrad g;
    g.dy = dy;
    g.dB = gr->dB; g.dC = gr->dC; g.du = gr->du; g.ddt = gr->ddt; g.dlam = gr->dlambda;
    g.G = (float*)w;
    g.pA = g.G + nG;
    g.pth = g.pA + (size_t)batch * s.N;
    if (s.bf16) blockscan_bwd_kernel<__nv_bfloat16><<<(unsigned)batch, bs_threads(s), 0, st>>>(s, g);
    else blockscan_bwd_kernel<float><<<(unsigned)batch, bs_threads(s), 0, st>>>(s, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("blockscan_bwd", e);
    if (gr->dA_log) bs_reduce_add<<<1, 64, 0, st>>>(g.pA, gr->dA_log, s.N, batch, s.N);
    if (gr->dtheta && s.N >= 2) bs_reduce_add<<<1, 32, 0, st>>>(g.pth, gr->dtheta, s.N / 2, batch, 32);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("blockscan reduce", e);
}
