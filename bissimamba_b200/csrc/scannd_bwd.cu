// scannd_bwd.cu -- exact Scan-A adjoint, parallel over the points of each
// wavefront level (any ndims <= 4; M a power of two <= 32, or a multiple of 32
// run as state tiles of 32, one launch per tile in order).
//
// Grid: one CTA per (item, channel group); a group is the RoPE pair
// (2g, 2g+1) when theta is set, one channel otherwise.  Threads are
// (point slot, state m): M consecutive lanes hold the M states of one point, so
// the sums over m (ddelta, dx, dlambda) are segmented warp shuffles.  Levels
// are walked from the last to the first (the host wavefront plan lists the
// points of every level); the points of a level are independent.  Each point
// PULLS its adjoint from its successors s = p + e_k:
//   g_h(p)  = C dy + R^T sum_k a_k(s) G(s)
//   g_Bu(p) = lam dt g_h(p) + sum_k beta(s)/n(s) G(s)
// where G(s) = g_h(s) was stored in a scratch array when level l+1 ran
// (visible after the level's __syncthreads), and the successor coefficients
// a_k(s), beta(s) are recomputed from delta(s), lambda(s).  No atomics: dA,
// dtheta and dlambda leave per-(item, group) partials that fixed-order
// reductions add into the outputs.  Reads B, C, h, x, delta, dy; writes G and
// accumulates dB, dC, ddelta, dx.  The states of a point are independent
// except for the sums over m (ddelta, dx, dlambda, dtheta), so M > 32 runs
// tiles of 32 states one after another: each tile adds its partial sums, in
// tile order (deterministic).
#include <vector>
#include "kmb_common.cuh"

namespace kmb {

int device_plan(const std::vector<long>& dims, long L, int** out, int* nlev, cudaStream_t st);
int set_error(const char* msg);
__global__ void reduce_rows_add(const float* __restrict__ part, float* __restrict__ out, long long count, long long n,
                                long long stride);
__global__ void reduce_lambda(const float* __restrict__ plam, float* __restrict__ dl, long long batch, int ngroups,
                              long long P);

struct WaveBwd {
    int D, M, has_lambda, fast, clamp;   // M: states of this launch (the tile)
    int MF, m0;                          // all states (the layout's stride) and the tile's first state
    float amin, deflam;
    long long P;
    int dims[4], strides[4];
    int nlev;
    const int* lev_start;
    const int* lev_pts;
    const int* nbr;   // per point: bit k = predecessor along axis k, bit 8 + k = successor along axis k
    const float *x, *A, *B, *C, *delta, *theta, *lambda, *h, *dy;
    float *dB, *dC, *ddelta, *dx;
    float *G, *pA, *pth, *plam;
};

// Two CTAs per SM (64 registers): the (item, channel-group) CTAs of a call are
// resident at once instead of running in two waves, and each SM hides twice the
// latency; the small register spill costs less than that gains.
template <int ND, bool ROPE>
__global__ void __launch_bounds__(512, 2) scan_bwd_wave(WaveBwd w) {
    const int D = w.D, M = w.M, MF = w.MF, m0 = w.m0;
    const int ngroups = ROPE ? (D + 1) / 2 : D;
    const int b = blockIdx.x / ngroups, g = blockIdx.x % ngroups;
    const int c0 = ROPE ? 2 * g : g;
    const int nc = (ROPE && c0 + 1 < D) ? 2 : 1;
    const bool rot = ROPE && nc == 2;
    const int tid = threadIdx.x, m = tid % M, slot = tid / M;
    const int nslots = blockDim.x / M;
    // item bases in 64-bit; indices inside an item in 32-bit (P * D * M < 2^31, checked by the launcher)
    const long long P = w.P, DM = (long long)D * MF;
    const int Pi = (int)P, DMi = D * MF;
    const float* __restrict__ x = w.x + b * P * D;
    const float* __restrict__ Bp = w.B + b * P * DM;
    const float* __restrict__ Cp = w.C + b * P * DM;
    const float* __restrict__ hp = w.h + b * P * DM;
    const float* __restrict__ dl = w.delta + b * ND * P * D;
    const float* __restrict__ dyp = w.dy + b * P * D;
    const float* __restrict__ lamp = w.has_lambda ? w.lambda + b * P : nullptr;
    float* __restrict__ G = w.G + b * P * DM;
    float* dBp = w.dB ? w.dB + b * P * DM : nullptr;
    float* dCp = w.dC ? w.dC + b * P * DM : nullptr;
    float* ddp = w.ddelta ? w.ddelta + b * ND * P * D : nullptr;
    float* dxp = w.dx ? w.dx + b * P * D : nullptr;

    float Ak[ND][2];
    bool clk[ND][2];
#pragma unroll
    for (int k = 0; k < ND; k++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const float a = (c < nc) ? w.A[((long long)k * D + c0 + c) * MF + m0 + m] : 0.0f;
            clk[k][c] = w.clamp && a > w.amin;
            Ak[k][c] = clk[k][c] ? w.amin : a;
        }
    float cth = 1.0f, sth = 0.0f;
    if (rot) {
        kmb_cos_sin(w.theta[g], &cth, &sth);
    }
    float gA[ND][2], gth = 0.0f;
#pragma unroll
    for (int k = 0; k < ND; k++) gA[k][0] = gA[k][1] = 0.0f;

    for (int lev = w.nlev - 1; lev >= 0; lev--) {
        const int beg = w.lev_start[lev], end = w.lev_start[lev + 1];
        for (int base = beg; base < end; base += nslots) {
            const int i = base + slot;
            const bool active = i < end;
            const int p = active ? w.lev_pts[i] : 0;
            // neighbour mask from the plan: no divisions per point
            const int nb = w.nbr[p];
            const int npred = __popc(nb & 0xff);
            float gdel[ND][2], gdt[2] = {0.f, 0.f}, gx[2] = {0.f, 0.f}, glam = 0.0f;
#pragma unroll
            for (int k = 0; k < ND; k++) gdel[k][0] = gdel[k][1] = 0.0f;
            if (active) {
                const float lam = lamp ? lamp[p] : w.deflam;
                // ---- pull from the successors
                float ah[2] = {0.f, 0.f}, ab[2] = {0.f, 0.f};
#pragma unroll
                for (int k = 0; k < ND; k++) {
                    if (!((nb >> (8 + k)) & 1)) continue;
                    const int s = p + w.strides[k];
                    const int ns = npred + (((nb >> k) & 1) ? 0 : 1);
                    const float lams = lamp ? lamp[s] : w.deflam;
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        if (c >= nc) continue;
                        float dts = 0.0f, sal = 0.0f, alk = 0.0f;
#pragma unroll
                        for (int k2 = 0; k2 < ND; k2++) {
                            const float dv = dl[(k2 * Pi + s) * D + c0 + c];
                            dts += dv;
                            const bool has = (k2 == k) || ((nb >> k2) & 1);   // successor's predecessor axes
                            if (has) {
                                const float a = kmb_exp(dv * Ak[k2][c], w.fast);
                                sal += a;
                                if (k2 == k) alk = a;
                            }
                        }
                        const float Gs = G[s * DMi + (c0 + c) * MF + m0 + m];
                        const float beta = (1.0f - lams) * dts * (sal / (float)ns);
                        ah[c] += alk * Gs;
                        ab[c] += beta / (float)ns * Gs;
                    }
                }
                float gh[2];
                const int o = p * DMi + c0 * MF + m0 + m;
                const float h0 = hp[o], h1 = rot ? hp[o + MF] : 0.0f;
                if (rot) {
                    gh[0] = cth * ah[0] + sth * ah[1];
                    gh[1] = -sth * ah[0] + cth * ah[1];
                    const float hat0 = cth * h0 - sth * h1, hat1 = sth * h0 + cth * h1;
                    gth += -ah[0] * hat1 + ah[1] * hat0;
                } else {
                    gh[0] = ah[0];
                    gh[1] = 0.0f;
                }
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    if (c >= nc) continue;
                    const int oc = o + c * MF;
                    const int d = c0 + c;
                    const float dyv = dyp[p * D + d];
                    const float hv = c ? h1 : h0;
                    gh[c] += Cp[oc] * dyv;
                    if (dCp) atomicAdd(&dCp[oc], dyv * hv);   // one addition: old + value
                    G[oc] = gh[c];
                    const float xv = x[p * D + d];
                    float dt = 0.0f;
                    float dk[ND];
#pragma unroll
                    for (int k = 0; k < ND; k++) {
                        dk[k] = dl[(k * Pi + p) * D + d];
                        dt += dk[k];
                    }
                    const float bv = Bp[oc];
                    const float bu = bv * xv;
                    const float gbu = lam * dt * gh[c] + ab[c];
                    if (dBp) atomicAdd(&dBp[oc], gbu * xv);
                    gx[c] = gbu * bv;
                    gdt[c] = lam * bu * gh[c];
                    glam += dt * bu * gh[c];
                    if (npred > 0) {
                        float sbu = 0.0f, sal = 0.0f, al[ND], hat[ND];
#pragma unroll
                        for (int k = 0; k < ND; k++) {
                            al[k] = 0.0f;
                            hat[k] = 0.0f;
                            if (!((nb >> k) & 1)) continue;
                            const int q = p - w.strides[k];
                            const int oq = q * DMi + c0 * MF + m0 + m;
                            al[k] = kmb_exp(dk[k] * Ak[k][c], w.fast);
                            sal += al[k];
                            sbu += Bp[oq + c * MF] * x[q * D + d];
                            if (rot) {
                                const float q0 = hp[oq], q1 = hp[oq + MF];
                                hat[k] = c ? sth * q0 + cth * q1 : cth * q0 - sth * q1;
                            } else {
                                hat[k] = hp[oq];
                            }
                        }
                        const float inv = 1.0f / (float)npred;
                        const float gbeta = sbu * inv * gh[c];
                        const float gsal = (1.0f - lam) * dt * inv * gbeta;
                        gdt[c] += (1.0f - lam) * sal * inv * gbeta;
                        glam -= dt * sal * inv * gbeta;
#pragma unroll
                        for (int k = 0; k < ND; k++) {
                            if (!((nb >> k) & 1)) continue;
                            const float z = dk[k] * Ak[k][c];
                            const float dz = kmb_dexp(z, al[k], w.fast) * (hat[k] * gh[c] + gsal);
                            gdel[k][c] += dz * Ak[k][c];
                            if (!clk[k][c]) gA[k][c] += dz * dk[k];
                        }
                    }
                }
            }
            // ---- sums over the M lanes of the point (segmented shuffles)
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                if (off >= M) break;
#pragma unroll
                for (int c = 0; c < 2; c++) {
#pragma unroll
                    for (int k = 0; k < ND; k++) gdel[k][c] += __shfl_xor_sync(0xffffffffu, gdel[k][c], off);
                    gdt[c] += __shfl_xor_sync(0xffffffffu, gdt[c], off);
                    gx[c] += __shfl_xor_sync(0xffffffffu, gx[c], off);
                }
                glam += __shfl_xor_sync(0xffffffffu, glam, off);
            }
            if (active && m == 0) {
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    if (c >= nc) continue;
                    const int d = c0 + c;
                    if (ddp)
#pragma unroll
                        for (int k = 0; k < ND; k++) atomicAdd(&ddp[(k * Pi + p) * D + d], gdel[k][c] + gdt[c]);
                    if (dxp) atomicAdd(&dxp[p * D + d], gx[c]);
                }
                w.plam[((long long)b * ngroups + g) * P + p] = glam;
            }
        }
        __syncthreads();
    }
    // ---- per-(item, group) partials of dA and dtheta (fixed-order block sums)
    __shared__ float red[512];
#pragma unroll
    for (int k = 0; k < ND; k++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            red[tid] = gA[k][c];
            __syncthreads();
            if (slot == 0 && c < nc) {
                float acc = 0.0f;
                for (int s2 = 0; s2 < nslots; s2++) acc += red[s2 * M + m];
                w.pA[(((long long)b * ND + k) * D + c0 + c) * MF + m0 + m] = acc;
            }
            __syncthreads();
        }
    if (rot) {
        red[tid] = gth;
        __syncthreads();
        if (tid == 0) {
            float acc = 0.0f;
            for (int t = 0; t < nslots * M; t++) acc += red[t];
            w.pth[(long long)b * (D / 2) + g] = acc;
        }
    }
}

template <int ND>
static cudaError_t wave_launch(const WaveBwd& w, bool rope, long long batch, int threads, cudaStream_t st) {
    const int ngroups = rope ? (w.D + 1) / 2 : w.D;
    const unsigned grid = (unsigned)(batch * ngroups);
    if (rope) scan_bwd_wave<ND, true><<<grid, threads, 0, st>>>(w);
    else scan_bwd_wave<ND, false><<<grid, threads, 0, st>>>(w);
    return cudaGetLastError();
}

size_t scan_bwd_wave_scratch_bytes(const ScanDesc& s) {
    const long long ngroups = s.rope ? (s.D + 1) / 2 : s.D;
    return ((size_t)s.batch * s.P * s.D * s.M + (size_t)s.batch * s.nd * s.D * s.M + (size_t)s.batch * (s.D / 2 + 1) +
            (size_t)s.batch * ngroups * s.P) * sizeof(float) + 4 * 256;
}

// cudaErrorNotSupported when the shape is outside the kernel's envelope.
cudaError_t launch_scan_bwd_wave(const ScanDesc& s, const float* dy, float* dA, float* dB, float* dC, float* ddelta,
                                 float* dlambda, float* dtheta, float* dx, void* scratch, cudaStream_t st) {
    const bool tiles = s.M > 32 && s.M % 32 == 0;
    if (s.nd < 1 || s.nd > 4 || (!tiles && (s.M > 32 || (s.M & (s.M - 1)) != 0)) || s.P > 0x7fffffffLL ||
        s.batch * s.D > 0x7fffffffLL ||
        s.P * s.D * s.M * s.nd >= (1LL << 31))   // 32-bit indexing inside an item
        return cudaErrorNotSupported;
    std::vector<long> dims(s.dims, s.dims + s.nd);
    int* plan = nullptr;
    int nlev = 0;
    if (device_plan(dims, (long)s.P, &plan, &nlev, st)) return cudaErrorUnknown;
    WaveBwd w;
    memset(&w, 0, sizeof w);
    const int Mt = tiles ? 32 : s.M;
    w.D = s.D; w.M = Mt; w.MF = s.M; w.m0 = 0; w.has_lambda = s.has_lambda; w.fast = s.fast_exp; w.clamp = s.clamp;
    w.amin = s.a_log_min; w.deflam = s.default_lambda; w.P = s.P;
    for (int k = 0; k < s.nd; k++) { w.dims[k] = (int)s.dims[k]; w.strides[k] = (int)s.strides[k]; }
    w.nlev = nlev; w.lev_start = plan; w.lev_pts = plan + nlev + 1;
    w.nbr = w.lev_pts + 2 * s.P;   // after the points and their in-level positions
    w.x = s.x; w.A = s.A; w.B = s.B; w.C = s.C; w.delta = s.delta; w.theta = s.theta; w.lambda = s.lambda;
    w.h = s.h; w.dy = dy; w.dB = dB; w.dC = dC; w.ddelta = ddelta; w.dx = dx;
    const long long ngroups = s.rope ? (s.D + 1) / 2 : s.D;
    auto align = [](char* p) { return (char*)(((uintptr_t)p + 255) & ~(uintptr_t)255); };
    char* c = align((char*)scratch);
    w.G = (float*)c; c = align(c + (size_t)s.batch * s.P * s.D * s.M * 4);
    w.pA = (float*)c; c = align(c + (size_t)s.batch * s.nd * s.D * s.M * 4);
    w.pth = (float*)c; c = align(c + (size_t)s.batch * (s.D / 2 + 1) * 4);
    w.plam = (float*)c;
    // threads: up to 512, whole points (multiples of the tile's M), at least one warp
    int threads = 512 / Mt * Mt;
    if (threads < 32) threads = 32;
    auto nb = [](long long n) { return (unsigned)((n + 255) / 256); };
    // one launch per state tile, in order; each adds its sums over m (ddelta, dx by one atomic addition per
    // element and launch; dtheta, dlambda through their partials, reduced before the next tile's launch)
    for (int m0 = 0; m0 < s.M; m0 += Mt) {
        w.m0 = m0;
        cudaError_t e;
        switch (s.nd) {
            case 1: e = wave_launch<1>(w, s.rope, s.batch, threads, st); break;
            case 2: e = wave_launch<2>(w, s.rope, s.batch, threads, st); break;
            case 3: e = wave_launch<3>(w, s.rope, s.batch, threads, st); break;
            default: e = wave_launch<4>(w, s.rope, s.batch, threads, st); break;
        }
        if (e != cudaSuccess) return e;
        if (dtheta && s.rope && s.D >= 2) {
            const long long cnt = s.D / 2;
            reduce_rows_add<<<nb(cnt), 256, 0, st>>>(w.pth, dtheta, cnt, s.batch, cnt);
        }
        if (dlambda) reduce_lambda<<<nb(s.batch * s.P), 256, 0, st>>>(w.plam, dlambda, s.batch, (int)ngroups, s.P);
    }
    if (dA) {
        const long long cnt = (long long)s.nd * s.D * s.M;
        reduce_rows_add<<<nb(cnt), 256, 0, st>>>(w.pA, dA, cnt, s.batch, cnt);
    }
    return cudaGetLastError();
}

}  // namespace kmb
