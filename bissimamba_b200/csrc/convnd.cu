// convnd.cu -- dense causal depthwise convND (reference src/convnd.c:396-531).
//
// The convolution has no dependence between output points, so the reference's
// level-by-level wavefront (one OpenMP region / one GPU launch per level) is
// replaced by a single launch over all (item, point, channel) triples.  The
// kernel is HBM-bound: 8 bytes per output (read input, write output) with the
// K^nd taps served from L1/L2.
//
// Forward sums taps in ascending kernel-linear order starting from the bias,
// the reference's order, so fp32 results match the reference bit-for-bit.
// Backward keeps the reference's overwrite semantics (dinput, dkernel, dbias
// are zeroed then filled, src/convnd.c:482-484): dinput is a gather with the
// mirrored taps (no atomics); dkernel/dbias are per-chunk partial sums in
// registers + shared memory, reduced across chunks in a fixed order
// (deterministic).
#include "kmb_common.cuh"

namespace kmb {

__global__ void __launch_bounds__(256) conv_fwd_kernel(ConvDesc c, const float* __restrict__ in,
                                                       const float* __restrict__ ker,
                                                       const float* __restrict__ bias,
                                                       float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = c.batch * c.P * c.D;
    if (i >= total) return;
    const int d = (int)(i % c.D);
    const long long bp = i / c.D;
    const long long p = bp % c.P;
    const long long b = bp / c.P;
    int oc[KMB_MAXND], kd[KMB_MAXND];
    for (int a = 0; a < c.nd; a++) {
        oc[a] = (int)((p / c.strides[a]) % c.dims[a]);
        kd[a] = 0;
    }
    const float* inb = in + b * c.P * c.D;
    float sum = bias ? bias[d] : 0.0f;
    for (int kl = 0; kl < c.V; kl++) {
        long long src = 0;
        bool ok = true;
        for (int a = 0; a < c.nd; a++) {
            const int sc = oc[a] - (c.K - 1 - kd[a]);
            if (sc < 0) { ok = false; break; }
            src += (long long)sc * c.strides[a];
        }
        if (ok) sum = __fmaf_rn(inb[src * c.D + d], ker[(long long)kl * c.D + d], sum);
        for (int a = c.nd - 1; a >= 0; a--) {  // kernel-linear increment, last axis fastest
            if (++kd[a] < c.K) break;
            kd[a] = 0;
        }
    }
    out[i] = sum;
}

// dinput[s,d] = sum_k dy[s + (K-1-k), d] * ker[k, d]   (gather form)
__global__ void __launch_bounds__(256) conv_bwd_input_kernel(ConvDesc c, const float* __restrict__ dy,
                                                             const float* __restrict__ ker,
                                                             float* __restrict__ din) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = c.batch * c.P * c.D;
    if (i >= total) return;
    const int d = (int)(i % c.D);
    const long long bp = i / c.D;
    const long long s = bp % c.P;
    const long long b = bp / c.P;
    int sc[KMB_MAXND], kd[KMB_MAXND];
    for (int a = 0; a < c.nd; a++) {
        sc[a] = (int)((s / c.strides[a]) % c.dims[a]);
        kd[a] = 0;
    }
    const float* dyb = dy + b * c.P * c.D;
    float acc = 0.0f;
    for (int kl = 0; kl < c.V; kl++) {
        long long o = 0;
        bool ok = true;
        for (int a = 0; a < c.nd; a++) {
            const long long oa = sc[a] + (c.K - 1 - kd[a]);
            if (oa >= c.dims[a]) { ok = false; break; }
            o += oa * c.strides[a];
        }
        if (ok) acc = __fmaf_rn(dyb[o * c.D + d], ker[(long long)kl * c.D + d], acc);
        for (int a = c.nd - 1; a >= 0; a--) {
            if (++kd[a] < c.K) break;
            kd[a] = 0;
        }
    }
    din[i] = acc;
}

// Partial dkernel / dbias over a chunk of (item, point) rows for 32 channels.
// block = 32 channel lanes x 8 row-warps; grid = (ceil(D/32), nchunks).
// part layout: [nchunks][V+1][D]  (row V holds dbias).
constexpr int kTapsPerPass = 28;

__global__ void __launch_bounds__(256) conv_bwd_kernel_partial(ConvDesc c, const float* __restrict__ in,
                                                               const float* __restrict__ dy,
                                                               float* __restrict__ part,
                                                               long long rows_per_chunk) {
    __shared__ float red[8][kTapsPerPass + 1][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int d = blockIdx.x * 32 + lane;
    const long long r0 = (long long)blockIdx.y * rows_per_chunk;
    const long long rows = c.batch * c.P;
    const long long r1 = min(r0 + rows_per_chunk, rows);
    const int npass = (c.V + kTapsPerPass - 1) / kTapsPerPass;
    for (int pass = 0; pass < npass; pass++) {
        const int t0 = pass * kTapsPerPass;
        const int nt = min(kTapsPerPass, c.V - t0);
        float acc[kTapsPerPass + 1];
#pragma unroll
        for (int t = 0; t <= kTapsPerPass; t++) acc[t] = 0.0f;
        if (d < c.D) {
            for (long long r = r0 + w; r < r1; r += 8) {
                const long long p = r % c.P, b = r / c.P;
                const float g = dy[r * c.D + d];
                if (pass == 0) acc[kTapsPerPass] += g;
                int oc[KMB_MAXND], kd[KMB_MAXND];
                int tmp = t0;
                for (int a = c.nd - 1; a >= 0; a--) {
                    kd[a] = tmp % c.K;
                    tmp /= c.K;
                }
                for (int a = 0; a < c.nd; a++) oc[a] = (int)((p / c.strides[a]) % c.dims[a]);
                const float* inb = in + b * c.P * c.D;
#pragma unroll
                for (int t = 0; t < kTapsPerPass; t++) {
                    if (t < nt) {
                        long long src = 0;
                        bool ok = true;
                        for (int a = 0; a < c.nd; a++) {
                            const int sc = oc[a] - (c.K - 1 - kd[a]);
                            if (sc < 0) { ok = false; break; }
                            src += (long long)sc * c.strides[a];
                        }
                        if (ok) acc[t] = __fmaf_rn(g, inb[src * c.D + d], acc[t]);
                        for (int a = c.nd - 1; a >= 0; a--) {
                            if (++kd[a] < c.K) break;
                            kd[a] = 0;
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t <= kTapsPerPass; t++) red[w][t][lane] = acc[t];
        __syncthreads();
        for (int t = w; t <= kTapsPerPass; t += 8) {
            float s = 0.0f;
            for (int j = 0; j < 8; j++) s += red[j][t][lane];
            if (d < c.D) {
                if (t < nt) part[((long long)blockIdx.y * (c.V + 1) + t0 + t) * c.D + d] = s;
                else if (t == kTapsPerPass && pass == 0)
                    part[((long long)blockIdx.y * (c.V + 1) + c.V) * c.D + d] = s;
            }
        }
        __syncthreads();
    }
}

// out[i] = sum_j part[j*stride + i]  (overwrite)
__global__ void reduce_rows_set(const float* __restrict__ part, float* __restrict__ out,
                                long long count, long long n, long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float acc = 0.0f;
    for (long long j = 0; j < n; j++) acc += part[j * stride + i];
    out[i] = acc;
}

static inline unsigned cblk(long long n, int t) { return (unsigned)((n + t - 1) / t); }
// ---------------------------------------------------------------------------
// Specialised kernels for ndims in {1,2,3}, K in {2,3,4}, D % 4 == 0: taps
// unrolled at compile time, four channels per thread (float4), tap validity
// from per-axis shift tests.  Same tap order as above (ascending kernel-linear
// index), so the forward stays bit-identical to the reference.
template <int ND, int K>
struct Taps {
    static constexpr int V = ND == 1 ? K : (ND == 2 ? K * K : K * K * K);
    // digit of axis a (0 = outermost) of kernel-linear index kl, last axis fastest
    __host__ __device__ static constexpr int digit(int kl, int a) {
        return ND == 1 ? kl : (ND == 2 ? (a == 0 ? kl / K : kl % K)
                                       : (a == 0 ? kl / (K * K) : (a == 1 ? (kl / K) % K : kl % K)));
    }
};

__device__ __forceinline__ void fma4(float4& acc, const float4 a, const float4 b) {
    acc.x = __fmaf_rn(a.x, b.x, acc.x);
    acc.y = __fmaf_rn(a.y, b.y, acc.y);
    acc.z = __fmaf_rn(a.z, b.z, acc.z);
    acc.w = __fmaf_rn(a.w, b.w, acc.w);
}

template <int ND, int K, bool BWD>
__global__ void __launch_bounds__(256) conv_tap_kernel(ConvDesc c, const float4* __restrict__ src,
                                                       const float4* __restrict__ ker,
                                                       const float4* __restrict__ bias, float4* __restrict__ dst) {
    // forward: dst[o] = bias + sum_k src[o - shift_k] * ker[k]
    // backward (dinput): dst[s] = sum_k src[s + shift_k] * ker[k]  (src = dy)
    // 32-bit index arithmetic: batch * P * D/4 < 2^31 (checked by the launcher)
    using T = Taps<ND, K>;
    const unsigned D4 = (unsigned)c.D >> 2, Pp = (unsigned)c.P;
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (unsigned)(c.batch * c.P) * D4) return;
    const unsigned d4 = i % D4;
    const unsigned bp = i / D4;
    const unsigned p = bp % Pp;
    int oc[3];
    unsigned st[3];
#pragma unroll
    for (int a = 0; a < ND; a++) {
        st[a] = (unsigned)c.strides[a];
        oc[a] = (int)((p / st[a]) % (unsigned)c.dims[a]);
    }
    float4 acc = BWD ? make_float4(0.f, 0.f, 0.f, 0.f) : (bias ? bias[d4] : make_float4(0.f, 0.f, 0.f, 0.f));
    const float4* s = src + (size_t)(bp - p) * D4;  // item base
#pragma unroll
    for (int kl = 0; kl < T::V; kl++) {
        bool ok = true;
        int off = (int)p;
#pragma unroll
        for (int a = 0; a < ND; a++) {
            const int sh = K - 1 - T::digit(kl, a);
            if (BWD) {
                ok = ok && (oc[a] + sh < (int)c.dims[a]);
                off += sh * (int)st[a];
            } else {
                ok = ok && (oc[a] >= sh);
                off -= sh * (int)st[a];
            }
        }
        if (ok) fma4(acc, s[(unsigned)off * D4 + d4], ker[kl * D4 + d4]);
    }
    dst[i] = acc;
}

// Streaming stencil along the outermost axis (V = K^ND <= 27): thread = (item,
// chunk of CH planes of axis 0, point of the remaining axes, 4 channels).  The K^ND
// kernel taps of the thread's channels sit in registers; each plane of the input
// (forward) or dy (backward, walked downwards) is loaded once as its K^(ND-1)
// neighbours and added into K rotating accumulators, the outputs of the K planes
// it reaches.  Loads per output fall from K^ND to K^(ND-1); the K-1 planes before
// a chunk are read to warm the accumulators up.  Summation order per output:
// by plane, then the remaining taps; fp32.
template <int ND, int K, bool BWD, int CH>
__global__ void __launch_bounds__(128) conv_stream_kernel(ConvDesc c, const float4* __restrict__ src,
                                                          const float4* __restrict__ ker,
                                                          const float4* __restrict__ bias, float4* __restrict__ dst,
                                                          int nchunks) {
    using T = Taps<ND, K>;
    constexpr int TR = T::V / K;   // taps of the remaining axes
    const int D4 = c.D >> 2;
    const int P0 = (int)c.dims[0];
    const long long Prest = c.P / P0;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= c.batch * nchunks * Prest * D4) return;
    const int d4 = (int)(i % D4);
    long long r = i / D4;
    const long long pr = r % Prest;
    r /= Prest;
    const int chunk = (int)(r % nchunks);
    const long long b = r / nchunks;
    int oc[3] = {0, 0, 0}, st[3] = {1, 1, 1};
#pragma unroll
    for (int a = 1; a < ND; a++) {
        st[a] = (int)c.strides[a];
        oc[a] = (int)((pr / st[a]) % c.dims[a]);
    }
    float4 kv[T::V];
#pragma unroll
    for (int kl = 0; kl < T::V; kl++) kv[kl] = ker[(long long)kl * D4 + d4];
    const float4 b0 = (!BWD && bias) ? bias[d4] : make_float4(0.f, 0.f, 0.f, 0.f);
    // the remaining-axes neighbour offsets of this point (in points), and which exist
    int roff[TR];   // points per item < 2^31 (checked by the launcher)
    bool rok[TR];
#pragma unroll
    for (int tr = 0; tr < TR; tr++) {
        int off = (int)pr;
        bool ok = true;
#pragma unroll
        for (int a = 1; a < ND; a++) {
            const int sh = K - 1 - T::digit(tr, a);   // digit of the remaining axes (axis 0 digit is 0 here)
            if (BWD) {
                ok = ok && (oc[a] + sh < c.dims[a]);
                off += sh * st[a];
            } else {
                ok = ok && (oc[a] >= sh);
                off -= sh * st[a];
            }
        }
        roff[tr] = ok ? off : 0;
        rok[tr] = ok;
    }
    const float4* s = src + b * c.P * D4;
    float4* o = dst + b * c.P * D4;
    const int lo = chunk * CH, hi = min(lo + CH, P0);   // outputs [lo, hi) of axis 0
    float4 acc[K];
#pragma unroll
    for (int j = 0; j < K; j++) acc[j] = b0;
    // forward walks planes lo-(K-1) .. hi-1 upwards; backward walks hi-1+(K-1) .. lo downwards
    const int first = BWD ? min(hi - 1 + (K - 1), P0 - 1) : max(lo - (K - 1), 0);
    const int last = BWD ? lo : hi - 1;
    const int step = BWD ? -1 : 1;
    for (int p0 = first;; p0 += step) {
        const long long pbase = (long long)p0 * Prest;
#pragma unroll
        for (int tr = 0; tr < TR; tr++) {
            if (!rok[tr]) continue;
            const float4 v = s[(pbase + roff[tr]) * D4 + d4];
#pragma unroll
            for (int sh0 = 0; sh0 < K; sh0++) fma4(acc[sh0], v, kv[(K - 1 - sh0) * TR + tr]);
        }
        // the output on this plane is complete
        const bool mine = BWD ? (p0 < hi) : (p0 >= lo);
        if (mine) o[((long long)p0 * Prest + pr) * D4 + d4] = acc[0];
#pragma unroll
        for (int j = 0; j < K - 1; j++) acc[j] = acc[j + 1];
        acc[K - 1] = b0;
        if (p0 == last) break;
    }
}

// dkernel / dbias partial sums: block = 32 float4 channel lanes x 8 row groups,
// grid = (ceil(D4 / 32), nchunks); part[chunk][V + 1][D].
template <int ND, int K>
__global__ void __launch_bounds__(256) conv_dk_tap_kernel(ConvDesc c, const float4* __restrict__ in,
                                                          const float4* __restrict__ dy, float4* __restrict__ part,
                                                          long long rows_per_chunk) {
    // taps are processed in passes of TP = K^(ND-1) (one value of the outermost
    // kernel digit per pass) to bound the register accumulators; pass 0 also
    // accumulates dbias
    using T = Taps<ND, K>;
    constexpr int NPASS = T::V > 16 ? K : 1;   // split only when the accumulators would not fit
    constexpr int TP = T::V / NPASS;
    __shared__ float4 red[8][32];
    const int D4 = c.D >> 2;
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int d4 = blockIdx.x * 32 + lane;
    // 32-bit index arithmetic: batch * P * D/4 < 2^31 (checked by the launcher)
    const unsigned r0 = (unsigned)(blockIdx.y * rows_per_chunk);
    const unsigned rows = (unsigned)(c.batch * c.P), Pp = (unsigned)c.P;
    const unsigned r1 = min(r0 + (unsigned)rows_per_chunk, rows);
    unsigned st[3];
#pragma unroll
    for (int a = 0; a < ND; a++) st[a] = (unsigned)c.strides[a];
#pragma unroll 1
    for (int pass = 0; pass < NPASS; pass++) {
        float4 acc[TP + 1];
#pragma unroll
        for (int t = 0; t <= TP; t++) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (d4 < D4) {
            for (unsigned r = r0 + grp; r < r1; r += 8) {
                const unsigned p = r % Pp;
                int oc[3];
#pragma unroll
                for (int a = 0; a < ND; a++) oc[a] = (int)((p / st[a]) % (unsigned)c.dims[a]);
                const float4 g = dy[r * D4 + d4];
                if (pass == 0) {
                    acc[TP].x += g.x; acc[TP].y += g.y; acc[TP].z += g.z; acc[TP].w += g.w;
                }
                const float4* s = in + (size_t)(r - p) * D4;
                const int sh0 = K - 1 - pass;  // shift of the outermost axis (NPASS == K)
                if (NPASS > 1 && oc[0] < sh0) continue;
#pragma unroll
                for (int t = 0; t < TP; t++) {
                    const int kl = pass * TP + t;
                    bool ok = true;
                    int off = NPASS > 1 ? (int)p - sh0 * (int)st[0] : (int)p;
#pragma unroll
                    for (int a = (NPASS > 1 ? 1 : 0); a < ND; a++) {
                        const int sh = K - 1 - T::digit(kl, a);
                        ok = ok && (oc[a] >= sh);
                        off -= sh * (int)st[a];
                    }
                    if (ok) fma4(acc[t], g, s[(unsigned)off * D4 + d4]);
                }
            }
        }
        for (int t = 0; t <= TP; t++) {
            if (t == TP && pass != 0) break;
            red[grp][lane] = acc[t];
            __syncthreads();
            if (grp == 0 && d4 < D4) {
                float4 v = red[0][lane];
                for (int j = 1; j < 8; j++) {
                    const float4 u = red[j][lane];
                    v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
                }
                const int slot = (t == TP) ? T::V : pass * TP + t;
                part[((long long)blockIdx.y * (T::V + 1) + slot) * D4 + d4] = v;
            }
            __syncthreads();
        }
    }
}

template <int ND, int K>
static cudaError_t conv_fast_impl(const ConvDesc& c, bool fwd, const float* in, const float* ker, const float* bias,
                                  float* out, const float* dy, float* din, float* dker, float* dbias, float* scratch,
                                  long long nch_max, cudaStream_t st) {
    const long long n4 = c.batch * c.P * (c.D / 4);
    const unsigned g4 = (unsigned)((n4 + 255) / 256);
    // streaming along axis 0 for 1D / 2D; 3D keeps the per-output gather (measured faster there)
    constexpr bool STREAM = ND <= 2 && Taps<ND, K>::V <= 27;
    if (c.batch * c.P * (c.D / 4) >= (1LL << 31)) return cudaErrorNotSupported;   // 32-bit indexing
    constexpr int CH = 8;   // planes of the outermost axis per thread
    const int nchunks = (int)((c.dims[0] + CH - 1) / CH);
    const long long ns = c.batch * nchunks * (c.P / c.dims[0]) * (c.D / 4);
    const unsigned gs = (unsigned)((ns + 127) / 128);
    if (fwd) {
        if constexpr (STREAM)
            conv_stream_kernel<ND, K, false, CH><<<gs, 128, 0, st>>>(c, (const float4*)in, (const float4*)ker,
                                                                     (const float4*)bias, (float4*)out, nchunks);
        else
            conv_tap_kernel<ND, K, false><<<g4, 256, 0, st>>>(c, (const float4*)in, (const float4*)ker,
                                                              (const float4*)bias, (float4*)out);
        return cudaGetLastError();
    }
    if constexpr (STREAM)
        conv_stream_kernel<ND, K, true, CH><<<gs, 128, 0, st>>>(c, (const float4*)dy, (const float4*)ker, nullptr,
                                                                (float4*)din, nchunks);
    else
        conv_tap_kernel<ND, K, true><<<g4, 256, 0, st>>>(c, (const float4*)dy, (const float4*)ker, nullptr,
                                                         (float4*)din);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long rows = c.batch * c.P;
    const int D4 = c.D / 4;
    const int dtiles = (D4 + 31) / 32;
    long long nch = (2LL * 148 * 4 + dtiles - 1) / dtiles;  // ~4 blocks per SM pair
    if (nch > rows) nch = rows;
    if (nch > nch_max) nch = nch_max;
    if (nch < 1) nch = 1;
    const long long rpc = (rows + nch - 1) / nch;
    dim3 grid(dtiles, (unsigned)nch);
    conv_dk_tap_kernel<ND, K><<<grid, 256, 0, st>>>(c, (const float4*)in, (const float4*)dy, (float4*)scratch, rpc);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const long long V = Taps<ND, K>::V, cnt = V * c.D;
    reduce_rows_set<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(scratch, dker, cnt, nch, (V + 1) * c.D);
    if (dbias)
        reduce_rows_set<<<(unsigned)((c.D + 255) / 256), 256, 0, st>>>(scratch + V * c.D, dbias, c.D, nch,
                                                                      (V + 1) * c.D);
    return cudaGetLastError();
}

// cudaErrorNotSupported when (ndims, K, D) is outside the specialised set.
static cudaError_t conv_fast(const ConvDesc& c, bool fwd, const float* in, const float* ker, const float* bias,
                             float* out, const float* dy, float* din, float* dker, float* dbias, float* scratch,
                             long long nch_max, cudaStream_t st) {
    if (c.D % 4 != 0) return cudaErrorNotSupported;
    const uintptr_t al = (uintptr_t)in | (uintptr_t)ker | (uintptr_t)(fwd ? out : din) | (uintptr_t)(fwd ? in : dy) |
                         (uintptr_t)(bias ? bias : ker);
    if (al & 15) return cudaErrorNotSupported;
#define KMB_CONV_CASE(ND_, K_) \
    if (c.nd == ND_ && c.K == K_) \
        return conv_fast_impl<ND_, K_>(c, fwd, in, ker, bias, out, dy, din, dker, dbias, scratch, nch_max, st);
    KMB_CONV_CASE(1, 2) KMB_CONV_CASE(1, 3) KMB_CONV_CASE(1, 4)
    KMB_CONV_CASE(2, 2) KMB_CONV_CASE(2, 3) KMB_CONV_CASE(2, 4)
    KMB_CONV_CASE(3, 2) KMB_CONV_CASE(3, 3) KMB_CONV_CASE(3, 4)
#undef KMB_CONV_CASE
    return cudaErrorNotSupported;
}


cudaError_t launch_conv_fused(const ConvDesc& c, int mode, const float* in, const float* ker, const float* bias,
                              float* out, const float* dy, float* din, float* dker, float* dbias, float* part,
                              long long nch_max, cudaStream_t st);
long long conv_fused_chunks(const ConvDesc& c, int mode);

cudaError_t launch_conv_fwd(const ConvDesc& c, const float* in, const float* ker, const float* bias,
                            float* out, cudaStream_t st) {
    cudaError_t ef = launch_conv_fused(c, 1, in, ker, bias, out, nullptr, nullptr, nullptr, nullptr, nullptr, 0, st);
    if (ef != cudaErrorNotSupported) return ef;
    ef = conv_fast(c, true, in, ker, bias, out, nullptr, nullptr, nullptr, nullptr, nullptr, 0, st);
    if (ef != cudaErrorNotSupported) return ef;
    conv_fwd_kernel<<<cblk(c.batch * c.P * c.D, 256), 256, 0, st>>>(c, in, ker, bias, out);
    return cudaGetLastError();
}

// forward and backward together: one fused launch when the shape allows it
cudaError_t launch_conv_both(const ConvDesc& c, const float* in, const float* ker, const float* bias, float* out,
                             const float* dy, float* din, float* dker, float* dbias, void* scratch, cudaStream_t st);

static long long conv_chunks(const ConvDesc& c) {
    const long long rows = c.batch * c.P;
    long long n = (rows + 255) / 256;  // >= 256 rows per chunk
    return n < 1 ? 1 : (n > 1024 ? 1024 : n);
}

size_t conv_bwd_scratch_bytes(const ConvDesc& c) {
    long long n = conv_chunks(c);
    const long long nf = conv_fused_chunks(c, 3);
    if (nf > n) n = nf;
    return (size_t)n * (c.V + 1) * c.D * sizeof(float);
}

cudaError_t launch_conv_bwd(const ConvDesc& c, const float* in, const float* ker, const float* dy,
                            float* din, float* dker, float* dbias, void* scratch, cudaStream_t st) {
    cudaError_t ef = launch_conv_fused(c, 2, in, ker, nullptr, nullptr, dy, din, dker, dbias, (float*)scratch,
                                       conv_fused_chunks(c, 2), st);
    if (ef != cudaErrorNotSupported) return ef;
    ef = conv_fast(c, false, in, ker, nullptr, nullptr, dy, din, dker, dbias, (float*)scratch,
                               conv_chunks(c), st);
    if (ef != cudaErrorNotSupported) return ef;
    conv_bwd_input_kernel<<<cblk(c.batch * c.P * c.D, 256), 256, 0, st>>>(c, dy, ker, din);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long nch = conv_chunks(c);
    const long long rows = c.batch * c.P;
    const long long rpc = (rows + nch - 1) / nch;
    float* part = (float*)scratch;
    dim3 grid(cblk(c.D, 32), (unsigned)nch);
    conv_bwd_kernel_partial<<<grid, 256, 0, st>>>(c, in, dy, part, rpc);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const long long cnt = (long long)c.V * c.D;
    reduce_rows_set<<<cblk(cnt, 256), 256, 0, st>>>(part, dker, cnt, nch, (long long)(c.V + 1) * c.D);
    if (dbias)
        reduce_rows_set<<<cblk(c.D, 256), 256, 0, st>>>(part + (long long)c.V * c.D, dbias, c.D, nch,
                                                       (long long)(c.V + 1) * c.D);
    return cudaGetLastError();
}



cudaError_t launch_conv_both(const ConvDesc& c, const float* in, const float* ker, const float* bias, float* out,
                             const float* dy, float* din, float* dker, float* dbias, void* scratch, cudaStream_t st) {
    cudaError_t e = launch_conv_fused(c, 3, in, ker, bias, out, dy, din, dker, dbias, (float*)scratch,
                                      conv_fused_chunks(c, 3), st);
    if (e != cudaErrorNotSupported) return e;
    if ((e = launch_conv_fwd(c, in, ker, bias, out, st)) != cudaSuccess) return e;
    return launch_conv_bwd(c, in, ker, dy, din, dker, dbias, scratch, st);
}

// ---------------------------------------------------------------------------
// convnd backward without any allocation.
//
// Some callers cannot allocate device memory: code that runs where
// cudaMalloc is forbidden or unsafe (inside a caller-owned memory pool or
// arena that must not grow, allocator hooks, real-time paths that may not
// take the allocator's locks).  For them the dkernel/dbias partial sums live
// in one fixed device array that is part of the loaded library.
//
// Limit: the partial-sum array holds kNoAllocScratchFloats floats (4 MiB);
// a call needs (K^ndims + 1) * D floats per row chunk and at least one chunk,
// so it is rejected when (K^ndims + 1) * D > kNoAllocScratchFloats.
// The array is shared by every call on a device and keeps the last call's
// contents; the kernels overwrite every entry they read, so nothing needs
// clearing.  Calls whose work overlaps on the GPU (different streams, or
// host threads without ordering) race on the array.
// ---------------------------------------------------------------------------
constexpr long long kNoAllocScratchFloats = 1 << 20;
static __device__ __align__(256) float g_conv_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
static float* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of the array on the current device.  The first call on a
// device resolves it (cudaGetSymbolAddress); make that first call before any
// stream capture.  The address is cached for the life of the process, so the
// entry point must not be used across a cudaDeviceReset of that device.
static cudaError_t noalloc_scratch_ptr(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
    float* p = __atomic_load_n(&g_noalloc_ptr[dev], __ATOMIC_ACQUIRE);
    if (!p) {
        e = cudaGetSymbolAddress((void**)&p, g_conv_noalloc_scratch);
        if (e != cudaSuccess) return e;
        __atomic_store_n(&g_noalloc_ptr[dev], p, __ATOMIC_RELEASE);
    }
    *out = p;
    return cudaSuccess;
}

static cudaError_t launch_conv_bwd_noalloc(const ConvDesc& c, const float* in, const float* ker, const float* dy,
                                           float* din, float* dker, float* dbias, cudaStream_t st) {
    const long long per_chunk = (long long)(c.V + 1) * c.D;
    if (per_chunk > kNoAllocScratchFloats) return cudaErrorInvalidValue;
    float* part = nullptr;
    cudaError_t e = noalloc_scratch_ptr(&part);
    if (e != cudaSuccess) return e;
    // the fast kernels first, with as many partial-sum chunks as the array holds
    e = launch_conv_fused(c, 2, in, ker, nullptr, nullptr, dy, din, dker, dbias, part,
                          kNoAllocScratchFloats / per_chunk, st);
    if (e != cudaErrorNotSupported) return e;
    cudaGetLastError();
    e = conv_fast(c, false, in, ker, nullptr, nullptr, dy, din, dker, dbias, part, kNoAllocScratchFloats / per_chunk, st);
    if (e != cudaErrorNotSupported) return e;
    cudaGetLastError();
    long long nch = conv_chunks(c);
    if (nch > kNoAllocScratchFloats / per_chunk) nch = kNoAllocScratchFloats / per_chunk;
    const long long rows = c.batch * c.P;
    const long long rpc = (rows + nch - 1) / nch;
    conv_bwd_input_kernel<<<cblk(c.batch * c.P * c.D, 256), 256, 0, st>>>(c, dy, ker, din);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    dim3 grid(cblk(c.D, 32), (unsigned)nch);
    conv_bwd_kernel_partial<<<grid, 256, 0, st>>>(c, in, dy, part, rpc);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const long long cnt = (long long)c.V * c.D;
    reduce_rows_set<<<cblk(cnt, 256), 256, 0, st>>>(part, dker, cnt, nch, per_chunk);
    if (dbias) reduce_rows_set<<<cblk(c.D, 256), 256, 0, st>>>(part + cnt, dbias, c.D, nch, per_chunk);
    return cudaGetLastError();
}

}  // namespace kmb

#include <cstdio>
#include <cstring>
#include "../../include/convnd.h"

static thread_local char tl_noalloc_err[160];

static bool noalloc_is_device(const void* p) {
    if (!p) return true;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

extern "C" const char* convnd_backward_noalloc_error(void) { return tl_noalloc_err; }

extern "C" int convnd_backward_noalloc(ConvNDParams* p, long batch, void* stream) {
    tl_noalloc_err[0] = 0;
    if (!p || !p->dims || p->ndims <= 0 || p->ndims > KMB_MAXND || p->D <= 0 || p->K <= 0 || batch < 1 ||
        !p->input || !p->kernel || !p->dy || !p->dinput || !p->dkernel) {
        snprintf(tl_noalloc_err, sizeof tl_noalloc_err, "invalid ConvNDParams");
        return -1;
    }
    const void* ptrs[] = {p->input, p->kernel, p->dy, p->dinput, p->dkernel, p->dbias};
    for (const void* q : ptrs)
        if (!noalloc_is_device(q)) {
            snprintf(tl_noalloc_err, sizeof tl_noalloc_err, "convnd_backward_noalloc needs device pointers");
            return -1;
        }
    kmb::ConvDesc c;
    memset(&c, 0, sizeof c);
    c.nd = (int)p->ndims;
    c.D = (int)p->D;
    c.K = (int)p->K;
    // (K^ndims + 1) * D must fit the array: check while multiplying, so a large K
    // or ndims cannot wrap the product past the limit
    const long long vmax = kmb::kNoAllocScratchFloats / p->D - 1;
    long long v = 1, P = 1;
    for (long i = 0; i < p->ndims; i++) {
        if (p->dims[i] <= 0) {
            snprintf(tl_noalloc_err, sizeof tl_noalloc_err, "invalid dims");
            return -1;
        }
        if (v > vmax / p->K) {
            snprintf(tl_noalloc_err, sizeof tl_noalloc_err,
                     "convnd_backward_noalloc: (K^ndims + 1) * D exceeds the %lld-float scratch limit",
                     kmb::kNoAllocScratchFloats);
            return -1;
        }
        v *= p->K;
        P *= p->dims[i];
    }
    c.V = (int)v;
    c.P = P;
    c.batch = batch;
    long long st = 1;
    for (int a = c.nd - 1; a >= 0; a--) {
        c.dims[a] = p->dims[a];
        c.strides[a] = st;
        st *= p->dims[a];
    }
    if ((long long)(c.V + 1) * c.D > kmb::kNoAllocScratchFloats) {
        snprintf(tl_noalloc_err, sizeof tl_noalloc_err,
                 "convnd_backward_noalloc: (K^ndims + 1) * D = %lld exceeds the %lld-float scratch limit",
                 (long long)(c.V + 1) * c.D, kmb::kNoAllocScratchFloats);
        return -1;
    }
    cudaError_t e = kmb::launch_conv_bwd_noalloc(c, p->input, p->kernel, p->dy, p->dinput, p->dkernel, p->dbias,
                                                 (cudaStream_t)stream);
    if (e != cudaSuccess) {
        snprintf(tl_noalloc_err, sizeof tl_noalloc_err, "convnd_backward_noalloc: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
