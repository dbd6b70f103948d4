/* qe_common.cuh: shared device helpers for the routed-MoE kernels (sm_100a). */
#ifndef QE_COMMON_CUH
#define QE_COMMON_CUH
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#define QE_CHECK(call)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) {                                                                    \
            fprintf(stderr, "qengine_b200: %s failed: %s (%s:%d)\n", #call, cudaGetErrorString(e_), \
                    __FILE__, __LINE__);                                                            \
            return -1;                                                                              \
        }                                                                                           \
    } while (0)

#define QE_FAIL(...)                                  \
    do {                                              \
        fprintf(stderr, "qengine_b200: " __VA_ARGS__); \
        fprintf(stderr, "\n");                        \
        return -1;                                    \
    } while (0)

static constexpr int QE_WARP = 32;

/* Raise a kernel's dynamic shared-memory limit once per (kernel, device), and only above the 48 KB default:
 * cudaFuncSetAttribute on every launch costs host time that a decode step cannot afford. */
#include <mutex>
#include <vector>
inline cudaError_t qe_set_smem(const void *kern, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    struct Entry { const void *k; int dev; size_t bytes; };
    static std::mutex mu;
    static std::vector<Entry> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    for (auto &d : done)
        if (d.k == kern && d.dev == dev && d.bytes >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done.push_back({kern, dev, bytes});
    return e;
}
static constexpr unsigned QE_FULL = 0xffffffffu;

__device__ __forceinline__ float qe_bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

/* ---------------------------------------------------------------------------------------------------
 * Exact single-precision exp, bit-identical to the host C library's expf on every input.
 *
 * The reference's softmax (engine/src/ops.c:29-42) calls the C library's expf, so routing weights can
 * only be reproduced bit for bit if the GPU evaluates the very same function. glibc (2.27 and later)
 * implements expf with the published table-driven method of Szabolcs Nagy (Arm optimized-routines,
 * 2017): x*N/ln2 = k + r with N = 32 and |r| <= 1/2, exp(x) = 2^(k/N) * 2^(r/N), 2^(r/N) by a cubic
 * polynomial, all in double precision, rounded once to float. On x86-64 CPUs with FMA the library
 * evaluates the argument reduction and the polynomial with fused multiply-adds; this function does
 * the same with DFMA. The 2^(i/32) table was computed here to 60 significant digits and rounded to
 * double; the polynomial coefficients are the method's published minimax constants.
 * tests/test_gpu_kernels.py compares it with the host expf over every negative float and every float in
 * [0, 88.72]; the same comparison on the CPU (this formula in C, with fma()) gave 0 mismatches over all
 * 2.1e9 negative floats.
 * ------------------------------------------------------------------------------------------------- */
/* In global memory (read through the read-only cache): the lanes of a warp index it differently, which
 * constant memory would serialise; 256 bytes, so a warp's lookups hit one or two L1 lines. */
__device__ const unsigned long long qe_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

__device__ __forceinline__ float qe_expf(float x) {
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32.0;
    const double kShift = 0x1.8p+52;
    const double kC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double kC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    /* branch-free: the main path is evaluated for every x (no input traps; results outside the range are
     * replaced below), so independent calls overlap */
    const double xd = (double)x;
    double kd = __fma_rn(kInvLn2N, xd, kShift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, kShift);
    const double r = __fma_rn(kInvLn2N, xd, -kd);
    const unsigned long long t = __ldg(qe_exp2_tab + (ki & 31ull)) + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double z = __fma_rn(kC0, r, kC1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(kC2, r, 1.0);
    y = __fma_rn(z, r2, y);
    y = __dmul_rn(y, s);
    float res = __double2float_rn(y);
    res = x > 0x1.62e42ep6f ? __int_as_float(0x7f800000) : res;   /* overflow */
    res = x < -0x1.9fe368p6f ? 0.0f : res;                         /* underflows to 0 (and -inf) */
    res = x != x ? x + x : res;                                     /* NaN */
    return res;
}

/* silu(g) * u exactly as engine/src/ops.c:16-21 evaluates it: g / (1 + expf(-g)) * u. */
__device__ __forceinline__ float qe_silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, qe_expf(-g))), u);
}

/* Same formula with CUDA's expf: for the SwiGLU inside the expert kernels, whose results are compared
 * within tolerance (routing, which must be bit-exact, always uses qe_expf). */
__device__ __forceinline__ float qe_silu_mul_fast(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

/* 1 / (1 + expf(-x)), engine/src/ops.c:23-27. */
__device__ __forceinline__ float qe_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, qe_expf(-x))); }

/* Split a float into three bf16 terms, x ~= hi + mid + lo, each the nearest bf16 of the remaining
 * residual (24 significant bits in total: the error is below 2^-24 |x| up to bf16 subnormals). */
__device__ __forceinline__ void qe_split3(float x, __nv_bfloat16 &hi, __nv_bfloat16 &mid, __nv_bfloat16 &lo) {
    hi = __float2bfloat16_rn(x);
    const float r1 = __fsub_rn(x, __bfloat162float(hi));
    mid = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, __bfloat162float(mid));
    lo = __float2bfloat16_rn(r2);
}

__device__ __forceinline__ uint32_t qe_pack_bf16(__nv_bfloat16 lo_half, __nv_bfloat16 hi_half) {
    return (uint32_t)__bfloat16_as_ushort(lo_half) | ((uint32_t)__bfloat16_as_ushort(hi_half) << 16);
}

#endif
