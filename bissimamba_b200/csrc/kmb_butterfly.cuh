// kmb_butterfly.cuh -- transposed butterfly reduction over the lanes of a warp
// (shared by the strip kernels).
#pragma once

namespace kmb {

// Transposed butterfly: v[NV] per lane -> lane holds the sum over its GS-lane
// group of value index idx_of(lane).  NV is a power of two <= GS.
template <int N>
struct Log2 {
    static constexpr int value = 1 + Log2<N / 2>::value;
};
template <>
struct Log2<1> {
    static constexpr int value = 0;
};

template <int NV, int GS>
__device__ __forceinline__ float butterfly(float (&v)[NV], int lane) {
    constexpr int LV = Log2<NV>::value, LG = Log2<GS>::value;
#pragma unroll
    for (int lvl = 0; lvl < LV; lvl++) {
        const int half = NV >> (lvl + 1);
        const int off = GS >> (lvl + 1);
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < NV / 2; i++) {
            if (i < half) {
                const float send = up ? v[i] : v[i + half];
                const float keep = up ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
    }
    float r = v[0];
#pragma unroll
    for (int lvl = LV; lvl < LG; lvl++) r += __shfl_xor_sync(0xffffffffu, r, GS >> (lvl + 1));
    return r;
}
// value index held by `lane` after butterfly<NV, GS>
template <int NV, int GS>
__device__ __forceinline__ int butterfly_index(int lane) {
    int idx = 0, n = NV, off = GS / 2;
    while (n > 1) {
        n >>= 1;
        if (lane & off) idx += n;
        off >>= 1;
    }
    return idx;
}

}  // namespace kmb
