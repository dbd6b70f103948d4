/* gemv_dev.cuh: lane-level helpers of the coalesced CUDA-core GEMVs (decode.cu).
 *
 * Codes follow the MLX affine layout of the reference (engine/src/qgroup.c: code j of a group at bit
 * (j % (32/bits))*bits of word j / (32/bits), LSB first).
 */
#ifndef QE_GEMV_DEV_CUH
#define QE_GEMV_DEV_CUH
#include <stdint.h>

#include "qe_common.cuh"

/* Code q as the float 1 + q/16 (4-bit) or 1 + q/256 (8-bit): the code's bits are the top mantissa bits, one
 * shift and one logic op. */
template <int BITS, int I>
__device__ __forceinline__ float code_v(uint32_t w) {
    constexpr int kTop = 23 - BITS;                 /* mantissa position of the code's lowest bit */
    constexpr int kSh = kTop - BITS * I;            /* left shift bringing code I there */
    constexpr uint32_t kMask = ((1u << BITS) - 1u) << kTop;
    const uint32_t s = kSh >= 0 ? (w << (kSh >= 0 ? kSh : 0)) : (w >> (kSh < 0 ? -kSh : 0));
    return __uint_as_float((s & kMask) | 0x3F800000u);
}

/* Transposed sum over the LPR lanes of a row of each of J values per lane: the levels pair lanes across lane
 * bit LPR/2, then LPR/4, ... 1; while values remain, each level halves them (a lane keeps the lower or upper half
 * by its bit), after that it adds the partner's single value. Lane l ends with value dg_index<LPR, J>(l). */
template <int LPR, int J>
__device__ __forceinline__ int dg_index(int lane) {
    int idx = 0;
#pragma unroll
    for (int o = LPR / 2, w = J / 2; o; o >>= 1, w >>= 1)
        if (w >= 1 && (lane & o)) idx += w;
    return idx;
}
/* whether lane l holds the one copy of its value that is written (its full-exchange bits are clear) */
template <int LPR, int J>
__device__ __forceinline__ bool dg_writer(int lane) {
    int mask = 0;
#pragma unroll
    for (int o = LPR / 2, w = J / 2; o; o >>= 1, w >>= 1)
        if (w < 1) mask |= o;
    return (lane & mask) == 0;
}
template <int LPR, int J>
__device__ __forceinline__ float dg_reduce(float (&v)[J], int lane) {
#pragma unroll
    for (int o = LPR / 2, w = J / 2; o; o >>= 1, w >>= 1) {
        if (w >= 1) {
            const bool up = lane & o;
#pragma unroll
            for (int j = 0; j < w; j++) {
                const float keep = up ? v[j + w] : v[j], give = up ? v[j] : v[j + w];
                v[j] = __fadd_rn(keep, __shfl_xor_sync(QE_FULL, give, o));
            }
        } else {
            v[0] = __fadd_rn(v[0], __shfl_xor_sync(QE_FULL, v[0], o));
        }
    }
    return v[0];
}

#endif
