/* route.cu: router logits, softmax, top-k and renormalisation, bit-exact with the reference.
 *
 * Reference: engine/src/moe_layer.c:29-37 (route), engine/src/ops.c:29-73 (op_softmax, op_topk).
 *
 * fp32 router (the benchmark configurations): the reference has no fp32 router, so the order of the
 * dot product is defined once and followed by the CPU checker (or_dot_f32 in oracle/moe_oracle.c):
 * 64-input fmaf chains starting from 0 in ascending index order, the chunk sums added in chunk order
 * to a total that starts at 0.0f. Both kernels below evaluate exactly that sequence of IEEE operations.
 * Quantized router (checkpoints): qmat_matvec's order (qmat.c:27-44, qgroup.c:48-53) without FMA.
 */
#include "qe_common.cuh"
#include "qe_kernels.h"
#include "route_dev.cuh"

namespace {

constexpr int kChunk = kRouterChunk;
constexpr int kMaxLaneChunks = kRouterLaneChunks;

/* Decode / small batch: one warp per router row (E routed rows + the shared gate row). */
__global__ void __launch_bounds__(128) router_gemv_f32_kernel(const float *__restrict__ W,
                                                              const float *__restrict__ bias,
                                                              const float *__restrict__ x, int T, int H, int E,
                                                              float *__restrict__ logits, int vec) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row > E) return;
    router_row_f32(W, bias, x, T, H, E, row, logits, vec);
}

/* Prefill: 64 router rows x 32 tokens per CTA, 128 threads, 4 rows x 4 tokens per thread. The K loop runs
 * in 64-input chunks; within a chunk every accumulator is an fmaf chain in ascending k, and at the end of
 * the chunk it is added to the running total: exactly or_dot_f32's order. Chunks are double-buffered in
 * shared memory, stored k-major ([k][row], [k][token]) so each k step is two broadcast 16-byte loads.
 * kSplit: the CTA (grid z) takes only kCG chunks and stores each chunk's chain value to
 * part[chunk][t][row]; router_sum_kernel then adds the chunks in order (same order, 8x more CTAs). */
constexpr int kGR = 64, kGT = 32, kCG = 2;
template <bool kSplit>
__global__ void __launch_bounds__(128) router_gemm_f32_kernel(const float *__restrict__ W,
                                                              const float *__restrict__ bias,
                                                              const float *__restrict__ x, int T, int H, int E,
                                                              float *__restrict__ logits, float *__restrict__ part) {
    __shared__ __align__(16) float Ws[2][kChunk][kGR];   /* [buf][k][row]   */
    __shared__ __align__(16) float Xs[2][kChunk][kGT];   /* [buf][k][token] */
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int r0 = blockIdx.x * kGR, t0 = blockIdx.y * kGT;
    const int Ep1 = E + 1;
    const int nch_all = (H + kChunk - 1) / kChunk;
    const int cbeg = kSplit ? blockIdx.z * kCG : 0;
    const int nch = kSplit ? min(nch_all, cbeg + kCG) : nch_all;   /* chunks [cbeg, nch) */
    /* loader mapping: W row = tid & 63, k quads (tid >> 6) + 2i (i < 8); X token = tid & 31, k quads
     * (tid >> 5) + 4i (i < 4). Consecutive lanes -> consecutive rows/tokens: conflict-free stores. */
    const int lr = tid & 63, lkq = tid >> 6, xr = tid & 31, xkq = tid >> 5;
    const bool wrow_ok = r0 + lr < Ep1, xrow_ok = t0 + xr < T;
    const float *wsrc = W + (size_t)(wrow_ok ? r0 + lr : 0) * H;
    const float *xsrc = x + (size_t)(xrow_ok ? t0 + xr : 0) * H;
    float4 wreg[8], xreg[4];
    auto load = [&](int c) {
        const int k0 = c * kChunk;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int k = k0 + 4 * (lkq + 2 * i);
            wreg[i] = (wrow_ok && k + 3 < H) ? __ldg(reinterpret_cast<const float4 *>(wsrc + k))
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = k0 + 4 * (xkq + 4 * i);
            xreg[i] = (xrow_ok && k + 3 < H) ? __ldg(reinterpret_cast<const float4 *>(xsrc + k))
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](int b) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int k = 4 * (lkq + 2 * i);
            Ws[b][k][lr] = wreg[i].x; Ws[b][k + 1][lr] = wreg[i].y;
            Ws[b][k + 2][lr] = wreg[i].z; Ws[b][k + 3][lr] = wreg[i].w;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int k = 4 * (xkq + 4 * i);
            Xs[b][k][xr] = xreg[i].x; Xs[b][k + 1][xr] = xreg[i].y;
            Xs[b][k + 2][xr] = xreg[i].z; Xs[b][k + 3][xr] = xreg[i].w;
        }
    };
    float total[4][4], acc[4][4];
    float2 acc2[4][2];   /* acc[i][2jj], acc[i][2jj+1] as pairs: independent chains in one paired fma */
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) total[i][j] = 0.0f;
    load(cbeg);
    store(0);
    __syncthreads();
    for (int c = cbeg; c < nch; c++) {
        const int b = (c - cbeg) & 1;
        if (c + 1 < nch) load(c + 1);
        const int kn = min(kChunk, H - c * kChunk);
#pragma unroll
        for (int i = 0; i < 4; i++) acc2[i][0] = acc2[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll 8
        for (int k = 0; k < kn; k++) {
            const float4 wv = *reinterpret_cast<const float4 *>(&Ws[b][k][ty * 4]);
            const float4 xv = *reinterpret_cast<const float4 *>(&Xs[b][k][tx * 4]);
            const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
            const float2 x01 = make_float2(xv.x, xv.y), x23 = make_float2(xv.z, xv.w);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 w2 = make_float2(wr[i], wr[i]);
                acc2[i][0] = __ffma2_rn(w2, x01, acc2[i][0]);
                acc2[i][1] = __ffma2_rn(w2, x23, acc2[i][1]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            acc[i][0] = acc2[i][0].x; acc[i][1] = acc2[i][0].y;
            acc[i][2] = acc2[i][1].x; acc[i][3] = acc2[i][1].y;
        }
        if constexpr (kSplit) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = r0 + ty * 4 + i;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int t = t0 + tx * 4 + j;
                    if (r < Ep1 && t < T) part[((size_t)c * T + t) * Ep1 + r] = acc[i][j];
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) total[i][j] = __fadd_rn(total[i][j], acc[i][j]);
        }
        if (c + 1 < nch) store(b ^ 1);
        __syncthreads();
    }
    if constexpr (!kSplit) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = r0 + ty * 4 + i;
            if (r >= Ep1) continue;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int t = t0 + tx * 4 + j;
                if (t >= T) continue;
                float l = total[i][j];
                if (bias && r < E) l = __fadd_rn(l, bias[r]);
                logits[(size_t)t * Ep1 + r] = l;
            }
        }
    }
}

/* Prefill, register-tiled: CTA = (64 router rows, 64 tokens[, kCG2 chunks of 64 inputs]), 64 threads, each
 * thread 8 rows (ty + 8i) x 8 tokens (tx + 8j). The W and x tiles of a chunk come by 16-byte cp.async into
 * shared memory as they lie in HBM ([row][k], [token][k], rows padded to kLds floats: the 4 rows and 8 tokens
 * a warp reads at one k quad fall in distinct banks), double-buffered. Per chunk every (row, token) value is
 * one fmaf chain in ascending k (or_dot_f32's order). kSplit (batches with few token tiles): the CTA takes
 * kCG2 chunks (grid z) and stores each chunk's value to part[chunk][row][token], router_sum2_kernel adds the
 * chunks in order; otherwise the CTA takes every chunk and adds them in order itself (no partial buffer).
 * Per k quad a thread loads 8 + 8 float4 for 256 FMAs (128 paired). */
constexpr int kGR2 = 64, kGT2 = 64, kCG2 = 2, kLds = kChunk + 4, kG2Threads = 64;

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <bool kSplit>
__global__ void __launch_bounds__(kG2Threads) router_gemm2_f32_kernel(const float *__restrict__ W,
                                                                      const float *__restrict__ bias,
                                                                      const float *__restrict__ x, int T, int H,
                                                                      int E, float *__restrict__ part,
                                                                      float *__restrict__ logits) {
    extern __shared__ __align__(16) float sm2[];
    float *Ws = sm2;                          /* [2][kGR2][kLds] */
    float *Xs = sm2 + 2 * kGR2 * kLds;        /* [2][kGT2][kLds] */
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int r0 = blockIdx.x * kGR2, t0 = blockIdx.y * kGT2;
    const int Ep1 = E + 1;
    const int nch_all = (H + kChunk - 1) / kChunk;
    const int cbeg = kSplit ? blockIdx.z * kCG2 : 0, cend = kSplit ? min(nch_all, cbeg + kCG2) : nch_all;
    float2 total[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int p2 = 0; p2 < 4; p2++) total[i][p2] = make_float2(0.0f, 0.0f);
    auto load = [&](int c, int b) {
        const int k0 = c * kChunk;
#pragma unroll
        for (int i = 0; i < kGR2 * kChunk / 4 / kG2Threads; i++) {
            const int idx = tid + kG2Threads * i, row = idx >> 4, q = idx & 15, k = k0 + 4 * q;
            const bool ok = r0 + row < Ep1 && k + 4 <= H;
            cp_async16_zfill((uint32_t)__cvta_generic_to_shared(Ws + (b * kGR2 + row) * kLds + 4 * q),
                             ok ? (const void *)(W + (size_t)(r0 + row) * H + k) : (const void *)W, ok ? 16u : 0u);
        }
#pragma unroll
        for (int i = 0; i < kGT2 * kChunk / 4 / kG2Threads; i++) {
            const int idx = tid + kG2Threads * i, tok = idx >> 4, q = idx & 15, k = k0 + 4 * q;
            const bool ok = t0 + tok < T && k + 4 <= H;
            cp_async16_zfill((uint32_t)__cvta_generic_to_shared(Xs + (b * kGT2 + tok) * kLds + 4 * q),
                             ok ? (const void *)(x + (size_t)(t0 + tok) * H + k) : (const void *)x, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load(cbeg, 0);
    for (int c = cbeg; c < cend; c++) {
        const int b = (c - cbeg) & 1;
        if (c + 1 < cend) {
            load(c + 1, b ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int kn = min(kChunk, H - c * kChunk);
        const float *wb = Ws + (b * kGR2 + ty) * kLds, *xb = Xs + (b * kGT2 + tx) * kLds;
        float2 acc[8][4];   /* [row i][token pair p]: tokens tx + 8*(2p), tx + 8*(2p+1); one fmaf chain each */
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int p2 = 0; p2 < 4; p2++) acc[i][p2] = make_float2(0.0f, 0.0f);
        for (int kq = 0; kq < kn; kq += 4) {
            float4 xv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) xv[j] = *reinterpret_cast<const float4 *>(xb + 8 * j * kLds + kq);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 wv = *reinterpret_cast<const float4 *>(wb + 8 * i * kLds + kq);
                const float w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const float2 w2 = make_float2(w[kk], w[kk]);
#pragma unroll
                    for (int p2 = 0; p2 < 4; p2++) {
                        const float4 &a = xv[2 * p2], &bq = xv[2 * p2 + 1];
                        const float xa = kk == 0 ? a.x : kk == 1 ? a.y : kk == 2 ? a.z : a.w;
                        const float xb2 = kk == 0 ? bq.x : kk == 1 ? bq.y : kk == 2 ? bq.z : bq.w;
                        acc[i][p2] = __ffma2_rn(w2, make_float2(xa, xb2), acc[i][p2]);
                    }
                }
            }
        }
        if constexpr (kSplit) {   /* part[c][row][token] */
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = r0 + ty + 8 * i;
                if (r >= Ep1) continue;
                float *dst = part + ((size_t)c * Ep1 + r) * T;
#pragma unroll
                for (int p2 = 0; p2 < 4; p2++) {
                    const int ta = t0 + tx + 8 * (2 * p2), tb = ta + 8;
                    if (ta < T) dst[ta] = acc[i][p2].x;
                    if (tb < T) dst[tb] = acc[i][p2].y;
                }
            }
        } else {                  /* chunks added in order */
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int p2 = 0; p2 < 4; p2++) total[i][p2] = __fadd2_rn(total[i][p2], acc[i][p2]);
        }
        __syncthreads();   /* buffer b is refilled two chunks later */
    }
    if constexpr (!kSplit) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = r0 + ty + 8 * i;
            if (r >= Ep1) continue;
            const float bv = bias && r < E ? bias[r] : 0.0f;
#pragma unroll
            for (int p2 = 0; p2 < 4; p2++) {
                const int ta = t0 + tx + 8 * (2 * p2), tb = ta + 8;
                if (ta < T) logits[(size_t)ta * Ep1 + r] = bias && r < E ? __fadd_rn(total[i][p2].x, bv) : total[i][p2].x;
                if (tb < T) logits[(size_t)tb * Ep1 + r] = bias && r < E ? __fadd_rn(total[i][p2].y, bv) : total[i][p2].y;
            }
        }
    }
}

/* logits[t][r] = (((0 + part[0][r][t]) + part[1][r][t]) + ...) + bias[r]: or_dot_f32's chunk order; one
 * thread per (r, t), consecutive threads consecutive tokens (coalesced reads of part). */
__global__ void router_sum2_kernel(const float *__restrict__ part, const float *__restrict__ bias, int nch, int T,
                                   int E, float *__restrict__ logits) {
    const int Ep1 = E + 1;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * Ep1) return;
    const int t = (int)(i % T), r = (int)(i / T);
    float tot = 0.0f;
    for (int c = 0; c < nch; c++) tot = __fadd_rn(tot, part[((size_t)c * Ep1 + r) * T + t]);
    if (bias && r < E) tot = __fadd_rn(tot, bias[r]);
    logits[(size_t)t * Ep1 + r] = tot;
}

/* logits[t][r] = (((0 + part[0][t][r]) + part[1][t][r]) + ...) + bias[r]: or_dot_f32's chunk order. */
__global__ void router_sum_kernel(const float *__restrict__ part, const float *__restrict__ bias, int nch, int T,
                                  int E, float *__restrict__ logits) {
    const int Ep1 = E + 1;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * Ep1) return;
    const int r = (int)(i % Ep1);
    float tot = 0.0f;
    for (int c = 0; c < nch; c++) tot = __fadd_rn(tot, part[(size_t)c * T * Ep1 + i]);
    if (bias && r < E) tot = __fadd_rn(tot, bias[r]);
    logits[i] = tot;
}

/* Quantized router in qmat_matvec's exact order: one warp per (row, token); lane g owns groups g, g+32,
 * ...: gsum_g and sum_q_g are sequential float sums (qmat.c:27-32, qgroup.c:48-53), then
 * t_g = scale*sum_q + bias*gsum and lane 0 adds the t_g in group order (qmat.c:41-44). */
__global__ void router_qmat_exact_kernel(QeQDev m, int row_base, const float *__restrict__ x, int T, int H,
                                         int ld, float *__restrict__ logits) {
    const int lane = threadIdx.x & 31;
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row = (int)(wid % m.rows), t = (int)(wid / m.rows);
    if (t >= T) return;
    const int gs = m.group_size, bits = m.bits, per = 32 / bits, ng = m.cols / gs;
    const uint32_t mask = (1u << bits) - 1u;
    const int wpr = m.cols * bits / 32, wpg = gs * bits / 32;
    const uint32_t *wp = m.w + (size_t)row * wpr;
    const float *xv = x + (size_t)t * H;
    float total = 0.0f;
    for (int g0 = 0; g0 < ng; g0 += 32) {
        const int g = g0 + lane;
        float tg = 0.0f;
        if (g < ng) {
            float gsum = 0.0f, sq = 0.0f;
            for (int i = 0; i < gs; i++) gsum = __fadd_rn(gsum, xv[g * gs + i]);
            const uint32_t *gw = wp + (size_t)g * wpg;
            for (int j = 0; j < gs; j++) {
                const float q = (float)((gw[j / per] >> ((j % per) * bits)) & mask);
                sq = __fadd_rn(sq, __fmul_rn(q, xv[g * gs + j]));
            }
            const float s = qe_bf16_to_f32(m.scales[(size_t)row * ng + g]);
            const float b = qe_bf16_to_f32(m.biases[(size_t)row * ng + g]);
            tg = __fadd_rn(__fmul_rn(s, sq), __fmul_rn(b, gsum));
        }
        const int nsrc = min(32, ng - g0);
        for (int src = 0; src < nsrc; src++) total = __fadd_rn(total, __shfl_sync(QE_FULL, tg, src));
    }
    if (lane == 0) logits[(size_t)t * ld + row_base + row] = total;
}

constexpr int kRouteWarps = 4;

/* Softmax + top-k + renormalisation: one warp per token (route_topk_warp). */
__global__ void __launch_bounds__(kRouteWarps * 32) route_topk_kernel(const float *__restrict__ logits, int ld,
                                                                      int T, int E, int k,
                                                                      int32_t *__restrict__ idx_out,
                                                                      float *__restrict__ score_out,
                                                                      float *__restrict__ probs_out) {
    extern __shared__ float smem[];
    const int w = threadIdx.x >> 5;
    const int t = blockIdx.x * kRouteWarps + w;
    if (t >= T) return;
    float *probs_s = smem + (size_t)w * 2 * E;   /* [E] */
    int *idx_s = reinterpret_cast<int *>(probs_s + E);
    route_topk_warp(logits + (size_t)t * ld, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
}

}  // namespace

int qe_launch_router_f32(const float *W, const float *bias, const float *x, int T, int H, int E, float *logits,
                         float *part, cudaStream_t s) {
    if (H > 32 * kMaxLaneChunks * kChunk) QE_FAIL("router: hidden %d too large", H);
    if (T <= 16) {
        const int rows = E + 1, warps_per_block = 4;
        const int vec = H % 4 == 0 && ((uintptr_t)W | (uintptr_t)x) % 16 == 0;
        router_gemv_f32_kernel<<<(rows + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(
            W, bias, x, T, H, E, logits, vec);
    } else {
        if (H % 4) QE_FAIL("router: hidden %d must be a multiple of 4", H);
        const int nch = (H + kChunk - 1) / kChunk;
        const int tiles = ((E + 1 + kGR2 - 1) / kGR2) * ((T + kGT2 - 1) / kGT2);
        const size_t smem = sizeof(float) * 2 * (kGR2 + kGT2) * kLds;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (((uintptr_t)W | (uintptr_t)x) % 16 == 0 && tiles >= 2 * sms) {
            /* enough tiles without splitting the inputs: every CTA adds its chunks itself */
            dim3 grid((E + 1 + kGR2 - 1) / kGR2, (T + kGT2 - 1) / kGT2);
            QE_CHECK(qe_set_smem((const void *)router_gemm2_f32_kernel<false>, smem));
            router_gemm2_f32_kernel<false><<<grid, kG2Threads, smem, s>>>(W, bias, x, T, H, E, nullptr, logits);
        } else if (part && ((uintptr_t)W | (uintptr_t)x) % 16 == 0) {
            dim3 grid((E + 1 + kGR2 - 1) / kGR2, (T + kGT2 - 1) / kGT2, (nch + kCG2 - 1) / kCG2);
            QE_CHECK(qe_set_smem((const void *)router_gemm2_f32_kernel<true>, smem));
            router_gemm2_f32_kernel<true><<<grid, kG2Threads, smem, s>>>(W, bias, x, T, H, E, part, nullptr);
            QE_CHECK(cudaGetLastError());
            const long long n = (long long)T * (E + 1);
            router_sum2_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, bias, nch, T, E, logits);
        } else if (part) {
            dim3 grid((E + 1 + kGR - 1) / kGR, (T + kGT - 1) / kGT, (nch + kCG - 1) / kCG);
            router_gemm_f32_kernel<true><<<grid, 128, 0, s>>>(W, bias, x, T, H, E, logits, part);
            QE_CHECK(cudaGetLastError());
            const long long n = (long long)T * (E + 1);
            router_sum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, bias, nch, T, E, logits);
        } else {
            dim3 grid((E + 1 + kGR - 1) / kGR, (T + kGT - 1) / kGT);
            router_gemm_f32_kernel<false><<<grid, 128, 0, s>>>(W, bias, x, T, H, E, logits, nullptr);
        }
    }
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_router_qmat(const QeQDev *router, const QeQDev *sh_router, const float *x, int T, int H, int E,
                          float *logits, cudaStream_t s) {
    const long long warps = (long long)router->rows * T;
    router_qmat_exact_kernel<<<(unsigned)((warps + 3) / 4), 128, 0, s>>>(*router, 0, x, T, H, E + 1, logits);
    QE_CHECK(cudaGetLastError());
    if (sh_router) {
        router_qmat_exact_kernel<<<(T + 3) / 4, 128, 0, s>>>(*sh_router, E, x, T, H, E + 1, logits);
        QE_CHECK(cudaGetLastError());
    }
    return 0;
}

int qe_launch_route_topk(const float *logits, int ld, int T, int E, int k, int32_t *idx, float *score,
                         float *probs, cudaStream_t s) {
    if (E < 1 || E > 32 * kMaxEPL) QE_FAIL("route: E=%d outside [1, %d]", E, 32 * kMaxEPL);
    if (k < 1 || k > 16 || k > E) QE_FAIL("route: top_k=%d outside [1, min(16, E)]", k);
    const size_t smem = (size_t)kRouteWarps * 2 * E * sizeof(float);
    route_topk_kernel<<<(T + kRouteWarps - 1) / kRouteWarps, kRouteWarps * 32, smem, s>>>(logits, ld, T, E, k, idx,
                                                                                        score, probs);
    QE_CHECK(cudaGetLastError());
    return 0;
}
