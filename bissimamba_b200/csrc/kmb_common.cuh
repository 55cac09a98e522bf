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

// Clamped cubic Taylor exponential of the reference (include/km_topology.h:52-56)
// or CUDA's accurate expf.
__device__ __forceinline__ float kmb_exp(float z, int fast) {
    if (fast) {
        z = fminf(fmaxf(z, -8.0f), 8.0f);
        return 1.0f + z + 0.5f * z * z + (1.0f / 6.0f) * z * z * z;
    }
    return expf(z);
}

// exp(z) = 2^(z log2 e) on the hardware base-2 exponential, with the rounding
// error of the product z * log2(e) recovered exactly by an FMA (plus the tail
// of log2 e beyond float precision) and applied as a first-order correction
// 2^(t + tl) ~ 2^t (1 + tl ln 2).  5 instructions, no branches; the error is
// that of ex2.approx (a couple of ulp), like expf's.  Results below 2^-126 are
// flushed to zero.
__device__ __forceinline__ float kmb_exp2c(float z) {
    const float kL2eHi = 1.44269502162933349609375f;   // float(log2 e)
    const float kL2eLo = 1.925963033500011e-08f;       // log2 e - kL2eHi
    const float t = __fmul_rn(z, kL2eHi);
    const float tl = __fmaf_rn(z, kL2eLo, __fmaf_rn(z, kL2eHi, -t));
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return __fmaf_rn(e, __fmul_rn(tl, 0.693147180559945309f), e);
}

// exp(z) as one hardware base-2 exponential of the rounded product
// z * log2(e): 2 instructions; adds up to ~|z log2 e| * 2^-24 relative error
// from the rounded product on top of ex2.approx's own (a few ulp for |z| < 4).
__device__ __forceinline__ float kmb_exp2r(float z) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(z, 1.44269502162933349609375f)));
    return e;
}

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
