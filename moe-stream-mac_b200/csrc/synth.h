/* synth.h: seeded synthetic inputs for the routed MoE block, bit-identical on the host and on the GPU.
 *
 * Every value is a pure function of (seed, stream, index), so a 123 GB expert stack can be generated in
 * HBM by a kernel while the CPU checker regenerates any subset of it with the same bits. Only integer
 * arithmetic, one IEEE float multiply and round-to-nearest-even bf16 packing are used, which both gcc
 * (no FMA contraction) and nvcc evaluate identically.
 *
 * Distributions (the benchmark configurations name N(0, sigma) for x, the router and the shared gate, and
 * scale = |N(0, 0.02)| / (2^(bits-1) - 0.5), bias = -(2^(bits-1) - 0.5) * scale for the affine experts):
 *   normal(sigma)  ~ sigma * sqrt(3) * (u0 + u1 + u2 + u3 - 2*65535) / 65536, u_i 16-bit uniform
 *                    (Irwin-Hall sum of four uniforms: mean 0, standard deviation sigma, bounded at 3.46 sigma)
 *   packed codes   a uniform 32-bit word per uint32 of the MLX layout, so every 4- or 8-bit code is uniform
 *   scale          bf16(|normal(0.02)| / 7.5 or / 127.5), bias = bf16(-7.5 * scale or -127.5 * scale)
 * The MLX affine layout itself (uint32 codes LSB first, bf16 scale/bias per group) follows
 * engine/include/qmat.h:3-11 of the reference.
 */
#ifndef QE_SYNTH_H
#define QE_SYNTH_H
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define SYN_HD __host__ __device__ __forceinline__
#else
#define SYN_HD static inline
#endif

/* Stream ids: one per tensor kind. Per-block and per-expert offsets are folded into the index. */
enum {
    SYN_X = 1,          /* activations x[T][hidden]                                  */
    SYN_ROUTER = 2,     /* fp32 router W[E][hidden]                                  */
    SYN_SHGATE = 3,     /* fp32 shared-expert gate w_sg[hidden]                      */
    SYN_PERM = 4,       /* rank -> expert permutation for skewed (Zipf) routing       */
    SYN_GATE = 8,       /* routed experts: codes use stream, scales use stream + 16   */
    SYN_UP = 9,
    SYN_DOWN = 10,
    SYN_SH_GATE = 11,   /* shared expert                                              */
    SYN_SH_UP = 12,
    SYN_SH_DOWN = 13,
    SYN_SCALE_OFS = 16
};

SYN_HD uint64_t syn_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* 64 random bits for element `i` of stream `stream` of block `block` under `seed`. */
SYN_HD uint64_t syn_hash(uint64_t seed, uint32_t block, uint32_t stream, uint64_t i) {
    const uint64_t key = syn_mix(seed ^ ((uint64_t)block << 32) ^ ((uint64_t)stream << 8));
    return syn_mix(key ^ syn_mix(i));
}

SYN_HD float syn_u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
SYN_HD uint32_t syn_f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* sigma_c = (float)(sigma * sqrt(3) / 65536), computed once by the caller. */
SYN_HD float syn_normal(uint64_t h, float sigma_c) {
    const int32_t s = (int32_t)(h & 0xffffu) + (int32_t)((h >> 16) & 0xffffu) +
                      (int32_t)((h >> 32) & 0xffffu) + (int32_t)(h >> 48) - 131070;
#ifdef __CUDA_ARCH__
    return __fmul_rn((float)s, sigma_c);
#else
    return (float)s * sigma_c;
#endif
}

/* float -> bf16 bit pattern, round to nearest even (NaN stays NaN). */
SYN_HD uint16_t syn_f32_to_bf16(float f) {
    uint32_t u = syn_f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

SYN_HD float syn_bf16_to_f32(uint16_t h) { return syn_u2f((uint32_t)h << 16); }

/* Packed code word `i` of a quantized tensor. */
SYN_HD uint32_t syn_code_word(uint64_t seed, uint32_t block, uint32_t stream, uint64_t i) {
    return (uint32_t)syn_hash(seed, block, stream, i);
}

/* Scale and bias of group `i`. scale_c = (float)(0.02 * sqrt(3) / 65536 / half_range),
 * neg_half_range = -(2^(bits-1) - 0.5) as a float (-7.5f or -127.5f). */
SYN_HD void syn_scale_bias(uint64_t seed, uint32_t block, uint32_t stream, uint64_t i, float scale_c,
                           float neg_half_range, uint16_t *scale, uint16_t *bias) {
    float s = syn_normal(syn_hash(seed, block, stream + SYN_SCALE_OFS, i), scale_c);
    s = s < 0.0f ? -s : s;
    const uint16_t sb = syn_f32_to_bf16(s);
#ifdef __CUDA_ARCH__
    const float b = __fmul_rn(neg_half_range, syn_bf16_to_f32(sb));
#else
    const float b = neg_half_range * syn_bf16_to_f32(sb);
#endif
    *scale = sb;
    *bias = syn_f32_to_bf16(b);
}

/* Host-side constants (double arithmetic, rounded once to float). */
static inline float syn_sigma_c(double sigma) { return (float)(sigma * 1.7320508075688772 / 65536.0); }
static inline float syn_scale_c(int bits) { return syn_sigma_c(0.02 / ((double)(1 << (bits - 1)) - 0.5)); }
static inline float syn_neg_half_range(int bits) { return (float)(-((double)(1 << (bits - 1)) - 0.5)); }

#endif
