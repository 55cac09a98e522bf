// kmb_common.cuh -- shared device/host helpers of libkmamba_b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define KMB_MAXND 16  // largest ndims the device kernels accept

// Device status codes written by kernels into the caller-visible status word.
enum KmbStatus : int {
    KMB_OK = 0,
    KMB_ERR_TIMEOUT_FULL = 1,   // a consumer gave up waiting for a staged tile
    KMB_ERR_TIMEOUT_EMPTY = 2,  // the producer gave up waiting for a free stage
    KMB_ERR_TIMEOUT_Y = 3,      // the reducer gave up waiting for the stage's states
};

// Scan-A problem description passed by value to the kernels.
struct ScanDesc {
    int nd;
    int D, M;
    int rope;            // theta != NULL
    int has_lambda;      // lambda != NULL
    int fast_exp;
    int clamp;
    int ex2;             // opt-in: alpha by one ex2.approx in the 2D strip kernel
    float a_log_min;
    float default_lambda;
    long long P;         // points per item
    long long batch;
    long long dims[KMB_MAXND];
    long long strides[KMB_MAXND];  // row-major point strides
    const float* x;
    const float* A;
    const float* B;
    const float* C;
    const float* delta;
    const float* theta;
    const float* lambda;
    float* h;
    float* y;
};

namespace kmb {
// convND problem description (batch of items, row-major points, channels last).
struct ConvDesc {
    int nd, D, K, V;          // V = K^nd
    long long P, batch;
    long long dims[KMB_MAXND];
    long long strides[KMB_MAXND];
};
}  // namespace kmb

// Clamped cubic Taylor exponential of the reference (include/km_topology.h:52-56)
// or CUDA's accurate expf.
__device__ __forceinline__ float kmb_exp(float z, int fast) {
    if (fast) {
        z = fminf(fmaxf(z, -8.0f), 8.0f);
        return 1.0f + z + 0.5f * z * z + (1.0f / 6.0f) * z * z * z;
    }
    return expf(z);
}

// cos and sin of a RoPE angle, evaluated in double precision and rounded once
// to float, so they are the correctly rounded values the reference's libm
// cosf / sinf return (the rotation is applied at every point of a recurrence:
// a one-ulp bias in it compounds over the levels).  Called once per tile.
__device__ __forceinline__ void kmb_cos_sin(float th, float* c, float* s) {
    double sd, cd;
    sincos((double)th, &sd, &cd);
    *c = (float)cd;
    *s = (float)sd;
}

// 2^w as one hardware base-2 exponential (ex2.approx, a few ulp for |w| < 4;
// results below 2^-126 flush to zero).  exp(delta * A) is evaluated as
// kmb_ex2(delta * (A log2 e)) with A log2 e rounded once per channel, so the
// argument carries ~|delta A log2 e| * 2^-23 relative error from two roundings:
// one multiply and one ex2 per exponential instead of expf's range-reduction
// sequence.
__device__ __forceinline__ float kmb_ex2(float w) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(w));
    return e;
}
constexpr float kKmbLog2e = 1.44269502162933349609375f;  // log2(e) rounded to float

// d/dz of kmb_exp given e = kmb_exp(z)
__device__ __forceinline__ float kmb_dexp(float z, float e, int fast) {
    if (fast) {
        if (z > 8.0f || z < -8.0f) return 0.0f;
        return 1.0f + z + 0.5f * z * z;
    }
    return e;
}

__device__ __forceinline__ float kmb_clampA(float a, int clamp, float amin) {
    return (clamp && a > amin) ? amin : a;
}
