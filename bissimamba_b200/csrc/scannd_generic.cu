// scannd_generic.cu -- Scan-A kernels for any shape (any ndims <= KMB_MAXND,
// any D, M, odd channel counts, unaligned sizes).
//
// Forward (reference src/scan_nd.c:103-201): one thread owns one recurrence
// lane (item b, channel group, state m), where a channel group is the RoPE pair
// (2g, 2g+1) when theta is set (the rotation couples the pair) and a single
// channel otherwise.  The thread walks the grid in row-major order, which is
// causal for the predecessor set {p - e_k}; predecessor states are re-read from
// the h it has already written and predecessor B*x products are recomputed
// (bit-identical to the reference's stored Bu_prev), so the kernel needs no
// scratch.  y = sum_m C h is formed afterwards by scan_y_kernel in ascending m,
// the reference's summation order.
//
// Backward: exact adjoint of the forward.  One thread owns (item, channel
// group) and all M states, visiting points in reverse row-major order and
// pushing adjoint contributions to the predecessors through zero-initialised
// scratch accumulators (private per thread, so no atomics).  Batch-shared
// gradients (dA, dtheta) and the cross-channel dlambda are written as per-item
// partials and reduced in a fixed order by small reduction kernels, so results
// are deterministic.
#include "kmb_common.cuh"

namespace kmb {

__device__ __forceinline__ void unravel(long long p, const ScanDesc& s, int* idx) {
    for (int k = 0; k < s.nd; k++) idx[k] = (int)((p / s.strides[k]) % s.dims[k]);
}

template <bool ROPE>
__global__ void __launch_bounds__(128) scan_fwd_generic(ScanDesc s) {
    const int D = s.D, M = s.M, nd = s.nd;
    const int ngroups = ROPE ? (D + 1) / 2 : D;
    const long long lane = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (lane >= s.batch * ngroups * M) return;
    const int m = (int)(lane % M);
    const long long t = lane / M;
    const int g = (int)(t % ngroups);
    const long long b = t / ngroups;
    const int d0 = ROPE ? 2 * g : g;
    const int nc = (ROPE && d0 + 1 < D) ? 2 : 1;
    const long long P = s.P;
    float cth = 1.0f, sth = 0.0f;
    if (ROPE && nc == 2) {
        const float th = s.theta[g];
        kmb_cos_sin(th, &cth, &sth);
    }
    int idx[KMB_MAXND];
    for (int k = 0; k < nd; k++) idx[k] = 0;
    const float* xb = s.x + b * P * D;
    const float* Bb = s.B + b * P * D * M;
    const float* db = s.delta + b * nd * P * D;
    float* hb = s.h + b * P * D * M;

    for (long long p = 0; p < P; p++) {
        const float lam = s.has_lambda ? s.lambda[b * P + p] : s.default_lambda;
        for (int c = 0; c < nc; c++) {
            const int d = d0 + c;
            const float xv = xb[p * D + d];
            float dt = 0.0f;
            for (int k = 0; k < nd; k++) dt = __fadd_rn(dt, db[((long long)k * P + p) * D + d]);
            const long long pdm = (p * D + d) * M + m;
            const float bu = __fmul_rn(Bb[pdm], xv);
            float buacc = 0.0f, dacc = 0.0f, hacc = 0.0f;
            int n = 0;
            for (int k = 0; k < nd; k++) {
                if (idx[k] > 0) {
                    const long long q = p - s.strides[k];
                    const float dta = db[((long long)k * P + p) * D + d];
                    const float av = kmb_clampA(s.A[((long long)k * D + d) * M + m], s.clamp, s.a_log_min);
                    const float al = kmb_exp(__fmul_rn(dta, av), s.fast_exp);
                    buacc = __fadd_rn(buacc, __fmul_rn(Bb[(q * D + d) * M + m], xb[q * D + d]));
                    dacc = __fadd_rn(dacc, al);
                    float hp;
                    if (ROPE && nc == 2) {
                        const float h0 = hb[(q * D + d0) * M + m];
                        const float h1 = hb[(q * D + d0 + 1) * M + m];
                        hp = (c == 0) ? (cth * h0 - sth * h1) : (sth * h0 + cth * h1);
                    } else {
                        hp = hb[(q * D + d) * M + m];
                    }
                    hacc = __fmaf_rn(al, hp, hacc);
                    n++;
                }
            }
            const float buavg = n > 0 ? __fdiv_rn(buacc, (float)n) : 0.0f;
            const float alavg = n > 0 ? __fdiv_rn(dacc, (float)n) : 0.0f;
            const float beta = (1.0f - lam) * dt * alavg;
            const float gamma = lam * dt;
            hb[pdm] = buavg * beta + bu * gamma + hacc;
        }
        for (int k = nd - 1; k >= 0; k--) {  // row-major increment
            if (++idx[k] < s.dims[k]) break;
            idx[k] = 0;
        }
    }
}

// y[b,p,d] = sum_m C h, ascending m (reference src/scan_nd.c:174).
__global__ void scan_y_kernel(const float* __restrict__ C, const float* __restrict__ h,
                              float* __restrict__ y, long long rows, int M) {
    const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float* c = C + r * M;
    const float* hh = h + r * M;
    float acc = 0.0f;
    for (int m = 0; m < M; m++) acc = __fmaf_rn(c[m], hh[m], acc);
    y[r] = acc;
}

struct BwdArgs {
    const float* dy;     // [b, P, D]
    float* dB;           // [b, P, D, M] or null
    float* dC;
    float* ddelta;       // [b, nd, P, D]
    float* dx;           // [b, P, D]
    float* acc_hat;      // scratch [b, P, D, M], zero
    float* acc_bu;       // scratch [b, P, D, M], zero
    float* pA;           // scratch [b, nd, D, M], zero
    float* pth;          // scratch [b, D/2]
    float* plam;         // scratch [b, ngroups, P]
};

template <bool ROPE>
__global__ void __launch_bounds__(64) scan_bwd_generic(ScanDesc s, BwdArgs a) {
    const int D = s.D, M = s.M, nd = s.nd;
    const int ngroups = ROPE ? (D + 1) / 2 : D;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= s.batch * ngroups) return;
    const int g = (int)(t % ngroups);
    const long long b = t / ngroups;
    const int d0 = ROPE ? 2 * g : g;
    const int nc = (ROPE && d0 + 1 < D) ? 2 : 1;
    const bool rot = ROPE && nc == 2;
    const long long P = s.P;
    float cth = 1.0f, sth = 0.0f;
    if (rot) {
        kmb_cos_sin(s.theta[g], &cth, &sth);
    }
    const float* xb = s.x + b * P * D;
    const float* Bb = s.B + b * P * D * M;
    const float* Cb = s.C + b * P * D * M;
    const float* db = s.delta + b * nd * P * D;
    const float* hb = s.h + b * P * D * M;
    const float* dyb = a.dy + b * P * D;
    float* ahb = a.acc_hat + b * P * D * M;
    float* abb = a.acc_bu + b * P * D * M;
    float* pAb = a.pA + b * nd * D * M;
    float dth = 0.0f;
    int idx[KMB_MAXND];
    for (int k = 0; k < nd; k++) idx[k] = (int)s.dims[k] - 1;

    for (long long p = P - 1; p >= 0; p--) {
        const float lam = s.has_lambda ? s.lambda[b * P + p] : s.default_lambda;
        float glam = 0.0f;
        float xv[2], dt[2], dyv[2], gdt[2] = {0.0f, 0.0f}, gx[2] = {0.0f, 0.0f};
        float gdel[2][KMB_MAXND];
        for (int c = 0; c < nc; c++) {
            const int d = d0 + c;
            xv[c] = xb[p * D + d];
            dyv[c] = dyb[p * D + d];
            float acc = 0.0f;
            for (int k = 0; k < nd; k++) {
                acc += db[((long long)k * P + p) * D + d];
                gdel[c][k] = 0.0f;
            }
            dt[c] = acc;
        }
        int n = 0;
        for (int k = 0; k < nd; k++) n += idx[k] > 0;
        for (int m = 0; m < M; m++) {
            float gh[2];
            if (rot) {
                const long long i0 = (p * D + d0) * M + m, i1 = i0 + M;
                const float a0 = ahb[i0], a1 = ahb[i1];
                gh[0] = cth * a0 + sth * a1;
                gh[1] = -sth * a0 + cth * a1;
                const float h0 = hb[i0], h1 = hb[i1];
                const float hat0 = cth * h0 - sth * h1, hat1 = sth * h0 + cth * h1;
                dth += -a0 * hat1 + a1 * hat0;
            } else {
                gh[0] = ahb[(p * D + d0) * M + m];
            }
            for (int c = 0; c < nc; c++) {
                const int d = d0 + c;
                const long long pdm = (p * D + d) * M + m;
                const float hv = hb[pdm];
                float g = gh[c] + Cb[pdm] * dyv[c];
                if (a.dC) a.dC[b * P * D * M + pdm] += dyv[c] * hv;
                const float bv = Bb[pdm];
                const float bu = bv * xv[c];
                const float gamma = lam * dt[c];
                const float gbu = gamma * g + abb[pdm];
                if (a.dB) a.dB[b * P * D * M + pdm] += gbu * xv[c];
                gx[c] += gbu * bv;
                const float ggam = bu * g;
                gdt[c] += lam * ggam;
                glam += dt[c] * ggam;
                if (n > 0) {
                    float sbu = 0.0f, sal = 0.0f;
                    float al[KMB_MAXND];
                    for (int k = 0; k < nd; k++) {
                        if (idx[k] == 0) continue;
                        const long long q = p - s.strides[k];
                        const float av = kmb_clampA(s.A[((long long)k * D + d) * M + m], s.clamp, s.a_log_min);
                        al[k] = kmb_exp(db[((long long)k * P + p) * D + d] * av, s.fast_exp);
                        sbu += Bb[(q * D + d) * M + m] * xb[q * D + d];
                        sal += al[k];
                    }
                    const float inv_n = 1.0f / (float)n;
                    const float beta = (1.0f - lam) * dt[c] * (sal * inv_n);
                    const float gbeta = (sbu * inv_n) * g;
                    const float gsal = (1.0f - lam) * dt[c] * inv_n * gbeta;
                    gdt[c] += (1.0f - lam) * (sal * inv_n) * gbeta;
                    glam -= dt[c] * (sal * inv_n) * gbeta;
                    for (int k = 0; k < nd; k++) {
                        if (idx[k] == 0) continue;
                        const long long q = p - s.strides[k];
                        const long long qdm = (q * D + d) * M + m;
                        float hat;
                        if (rot) {
                            const float h0 = hb[(q * D + d0) * M + m], h1 = hb[(q * D + d0 + 1) * M + m];
                            hat = (c == 0) ? (cth * h0 - sth * h1) : (sth * h0 + cth * h1);
                        } else {
                            hat = hb[qdm];
                        }
                        const float araw = s.A[((long long)k * D + d) * M + m];
                        const bool clamped = s.clamp && araw > s.a_log_min;
                        const float av = clamped ? s.a_log_min : araw;
                        const float dta = db[((long long)k * P + p) * D + d];
                        const float z = dta * av;
                        const float gal = hat * g + gsal;
                        const float dz = kmb_dexp(z, al[k], s.fast_exp) * gal;
                        gdel[c][k] += dz * av;
                        if (!clamped) pAb[((long long)k * D + d) * M + m] += dz * dta;
                        ahb[qdm] += al[k] * g;
                        abb[qdm] += beta * inv_n * g;
                    }
                }
            }
        }
        for (int c = 0; c < nc; c++) {
            const int d = d0 + c;
            if (a.ddelta)
                for (int k = 0; k < nd; k++)
                    a.ddelta[((b * nd + k) * P + p) * D + d] += gdel[c][k] + gdt[c];
            if (a.dx) a.dx[(b * P + p) * D + d] += gx[c];
        }
        a.plam[(b * ngroups + g) * P + p] = glam;
        for (int k = nd - 1; k >= 0; k--) {  // row-major decrement
            if (--idx[k] >= 0) break;
            idx[k] = (int)s.dims[k] - 1;
        }
    }
    if (rot) a.pth[b * (D / 2) + g] = dth;
}

// out[i] += sum_{j<n} part[j*stride + i]  (fixed order => deterministic)
__global__ void reduce_rows_add(const float* __restrict__ part, float* __restrict__ out,
                                long long count, long long n, long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float acc = 0.0f;
    for (long long j = 0; j < n; j++) acc += part[j * stride + i];
    out[i] += acc;
}

// dlambda[b,p] += sum_g plam[b,g,p]
__global__ void reduce_lambda(const float* __restrict__ plam, float* __restrict__ dl,
                              long long batch, int ngroups, long long P) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * P) return;
    const long long b = i / P, p = i % P;
    float acc = 0.0f;
    for (int g = 0; g < ngroups; g++) acc += plam[(b * ngroups + g) * P + p];
    dl[i] += acc;
}

// ------------------------------------------------------------ host launchers
static inline unsigned nblk(long long n, int t) { return (unsigned)((n + t - 1) / t); }

cudaError_t launch_scan_fwd_generic(const ScanDesc& s, cudaStream_t st) {
    const int ngroups = s.rope ? (s.D + 1) / 2 : s.D;
    const long long lanes = s.batch * ngroups * s.M;
    if (s.rope) scan_fwd_generic<true><<<nblk(lanes, 128), 128, 0, st>>>(s);
    else scan_fwd_generic<false><<<nblk(lanes, 128), 128, 0, st>>>(s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long rows = s.batch * s.P * s.D;
    scan_y_kernel<<<nblk(rows, 256), 256, 0, st>>>(s.C, s.h, s.y, rows, s.M);
    return cudaGetLastError();
}

size_t scan_bwd_generic_scratch_bytes(const ScanDesc& s) {
    const long long ngroups = s.rope ? (s.D + 1) / 2 : s.D;
    const long long st = s.batch * s.P * s.D * s.M;
    size_t n = 2 * st + s.batch * s.nd * s.D * s.M + s.batch * (s.D / 2 + 1) + s.batch * ngroups * s.P;
    return n * sizeof(float) + 4 * 256;
}

// scratch must hold scan_bwd_generic_scratch_bytes(s) bytes.
cudaError_t launch_scan_bwd_generic(const ScanDesc& s, const float* dy, float* dA, float* dB,
                                    float* dC, float* ddelta, float* dlambda, float* dtheta,
                                    float* dx, void* scratch, cudaStream_t st) {
    const long long ngroups = s.rope ? (s.D + 1) / 2 : s.D;
    const long long nst = s.batch * s.P * s.D * s.M;
    auto align = [](char* p) { return (char*)(((uintptr_t)p + 255) & ~(uintptr_t)255); };
    char* w = align((char*)scratch);
    BwdArgs a;
    a.dy = dy; a.dB = dB; a.dC = dC; a.ddelta = ddelta; a.dx = dx;
    a.acc_hat = (float*)w; w = align(w + nst * 4);
    a.acc_bu = (float*)w; w = align(w + nst * 4);
    a.pA = (float*)w; w = align(w + s.batch * s.nd * s.D * s.M * 4);
    a.pth = (float*)w; w = align(w + s.batch * (s.D / 2 + 1) * 4);
    a.plam = (float*)w;
    const size_t zero_bytes = (size_t)((char*)a.pth - (char*)a.acc_hat);
    cudaError_t e = cudaMemsetAsync(a.acc_hat, 0, zero_bytes, st);
    if (e != cudaSuccess) return e;
    const long long thr = s.batch * ngroups;
    if (s.rope) scan_bwd_generic<true><<<nblk(thr, 64), 64, 0, st>>>(s, a);
    else scan_bwd_generic<false><<<nblk(thr, 64), 64, 0, st>>>(s, a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (dA) {
        const long long cnt = (long long)s.nd * s.D * s.M;
        reduce_rows_add<<<nblk(cnt, 256), 256, 0, st>>>(a.pA, dA, cnt, s.batch, cnt);
    }
    if (dtheta && s.rope && s.D >= 2) {
        const long long cnt = s.D / 2;
        reduce_rows_add<<<nblk(cnt, 256), 256, 0, st>>>(a.pth, dtheta, cnt, s.batch, cnt);
    }
    if (dlambda)
        reduce_lambda<<<nblk(s.batch * s.P, 256), 256, 0, st>>>(a.plam, dlambda, s.batch, (int)ngroups, s.P);
    return cudaGetLastError();
}

}  // namespace kmb
