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

/* Prefill, register-tiled: CTA = (64 router rows, 64 tokens[, cg chunks of 64 inputs]), 64 threads, each
 * thread 8 rows (ty + 8i) x 8 tokens (tx + 8j). The W and x tiles of a chunk come by 16-byte cp.async into
 * shared memory as they lie in HBM ([row][k], [token][k], rows padded to kLds floats: the 4 rows and 8 tokens
 * a warp reads at one k quad fall in distinct banks), double-buffered when the CTA takes more than one chunk.
 * Per chunk every (row, token) value is one fmaf chain in ascending k (or_dot_f32's order). kSplit (batches
 * with few token tiles): the CTA takes cg chunks (grid z) and stores each chunk's value to
 * part[chunk][row][token], router_sum2_kernel adds the chunks in order; otherwise the CTA takes every chunk and
 * adds them in order itself (no partial buffer). Per k quad a thread loads 8 + 8 float4 for 256 FMAs (128
 * paired). When the router has 64n + 1 rows (E = 256 routed rows plus the shared-expert gate row), the CTAs of
 * the last row tile also compute row xrow (the gate row), thread i for token i of the tile, instead of a fifth
 * row tile of one row. */
constexpr int kGR2 = 64, kGT2 = 64, kLds = kChunk + 4, kG2Threads = 64, kWRows2 = kGR2 + 1;

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <bool kSplit>
__global__ void __launch_bounds__(kG2Threads, kSplit ? 6 : 1) router_gemm2_f32_kernel(const float *__restrict__ W,
                                                                      const float *__restrict__ bias,
                                                                      const float *__restrict__ x, int T, int H,
                                                                      int E, float *__restrict__ part,
                                                                      float *__restrict__ logits, int cg, int nbuf,
                                                                      int xrow) {
    extern __shared__ __align__(16) float sm2[];
    float *Ws = sm2;                              /* [nbuf][kWRows2][kLds] */
    float *Xs = sm2 + nbuf * kWRows2 * kLds;      /* [nbuf][kGT2][kLds] */
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int r0 = blockIdx.x * kGR2, t0 = blockIdx.y * kGT2;
    const int Ep1 = E + 1;
    const int xr = blockIdx.x == gridDim.x - 1 ? xrow : -1;   /* this CTA's extra row, or -1 */
    const int nch_all = (H + kChunk - 1) / kChunk;
    const int cbeg = kSplit ? blockIdx.z * cg : 0, cend = kSplit ? min(nch_all, cbeg + cg) : nch_all;
    float2 total[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int p2 = 0; p2 < 4; p2++) total[i][p2] = make_float2(0.0f, 0.0f);
    float totx = 0.0f;   /* extra row, token t0 + tid */
    auto load = [&](int c, int b) {
        const int k0 = c * kChunk;
#pragma unroll
        for (int i = 0; i < kGR2 * kChunk / 4 / kG2Threads; i++) {
            const int idx = tid + kG2Threads * i, row = idx >> 4, q = idx & 15, k = k0 + 4 * q;
            const bool ok = r0 + row < Ep1 && k + 4 <= H;
            cp_async16_zfill((uint32_t)__cvta_generic_to_shared(Ws + (b * kWRows2 + row) * kLds + 4 * q),
                             ok ? (const void *)(W + (size_t)(r0 + row) * H + k) : (const void *)W, ok ? 16u : 0u);
        }
        if (xr >= 0 && tid < kChunk / 4) {
            const int k = k0 + 4 * tid;
            const bool ok = k + 4 <= H;
            cp_async16_zfill((uint32_t)__cvta_generic_to_shared(Ws + (b * kWRows2 + kGR2) * kLds + 4 * tid),
                             ok ? (const void *)(W + (size_t)xr * H + k) : (const void *)W, ok ? 16u : 0u);
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
        const int b = nbuf == 2 ? (c - cbeg) & 1 : 0;
        if (nbuf == 2 && c + 1 < cend) {
            load(c + 1, b ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int kn = min(kChunk, H - c * kChunk);
        const float *wb = Ws + (b * kWRows2 + ty) * kLds, *xb = Xs + (b * kGT2 + tx) * kLds;
        const float *wx = Ws + (b * kWRows2 + kGR2) * kLds, *xt = Xs + (b * kGT2 + tid) * kLds;
        float2 acc[8][4];   /* [row i][token pair p]: tokens tx + 8*(2p), tx + 8*(2p+1); one fmaf chain each */
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int p2 = 0; p2 < 4; p2++) acc[i][p2] = make_float2(0.0f, 0.0f);
        float ax = 0.0f;
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
            if (xr >= 0) {
                const float4 wv = *reinterpret_cast<const float4 *>(wx + kq);
                const float4 xq = *reinterpret_cast<const float4 *>(xt + kq);
                ax = __fmaf_rn(wv.x, xq.x, ax);
                ax = __fmaf_rn(wv.y, xq.y, ax);
                ax = __fmaf_rn(wv.z, xq.z, ax);
                ax = __fmaf_rn(wv.w, xq.w, ax);
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
            if (xr >= 0 && t0 + tid < T) part[((size_t)c * Ep1 + xr) * T + t0 + tid] = ax;
        } else {                  /* chunks added in order */
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int p2 = 0; p2 < 4; p2++) total[i][p2] = __fadd2_rn(total[i][p2], acc[i][p2]);
            totx = __fadd_rn(totx, ax);
        }
        __syncthreads();   /* buffer b is refilled by the next chunk's load */
        if (nbuf == 1 && c + 1 < cend) load(c + 1, 0);
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
        if (xr >= 0 && t0 + tid < T)
            logits[(size_t)(t0 + tid) * Ep1 + xr] = bias && xr < E ? __fadd_rn(totx, bias[xr]) : totx;
    }
}

/* Prefill router GEMM on paired FMAs whose operands come from shared memory as register pairs: the router
 * weights are stored once per handle as Wd[k][row][2] (each value twice: the broadcast half of the pair) and
 * the batch is transposed per call to xt[k][token] (consecutive tokens: the other half). CTA = 64 router rows x
 * 64 tokens [x cg chunks of 64 inputs], 64 threads, thread (tx, ty): rows 32a + 4ty + i and tokens
 * 32b + 4tx + 2p (+1), a, b, p in {0, 1}, i < 4: 32 accumulator pairs. Inputs arrive in stages of 16 k by
 * cp.async through a ring of 3 (37 KB). Per chunk every (row, token) value is one fmaf chain in ascending k
 * (or_dot_f32's order); the chunks go to part[chunk][row][token] (kSplit) or are added in order in registers.
 * When Wd holds the first E rows of E + 1 = 64n + 1, thread i of the last row tile's CTAs also computes the
 * gate row E (read from W) for token i of the tile. */
constexpr int kG3Rows = 64, kG3Toks = 64, kG3K = 16, kG3Stages = 3, kG3Threads = 64;
constexpr int kG3WdFloats = kG3K * kG3Rows * 2, kG3XFloats = kG3K * kG3Toks;
constexpr int kG3StageFloats = kG3WdFloats + kG3XFloats + kG3K;

template <bool kSplit>
__global__ void __launch_bounds__(kG3Threads, kSplit ? 6 : 4)
    router_gemm3_f32_kernel(const float *__restrict__ Wd, int R, const float *__restrict__ W,
                            const float *__restrict__ bias, const float *__restrict__ xt, int Tp, int T, int H,
                            int E, float *__restrict__ part, float *__restrict__ logits, int cg, int xrow) {
    __shared__ __align__(16) float sm3[kG3Stages * kG3StageFloats];
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int r0 = blockIdx.x * kG3Rows, t0 = blockIdx.y * kG3Toks;
    const int Ep1 = E + 1;
    const int xr = blockIdx.x == gridDim.x - 1 ? xrow : -1;   /* the gate row, or -1 */
    const int nch_all = (H + kChunk - 1) / kChunk;
    const int cbeg = kSplit ? blockIdx.z * cg : 0, cend = kSplit ? min(nch_all, cbeg + cg) : nch_all;
    const int kbeg = cbeg * kChunk, kend = min(H, cend * kChunk);
    const int nst = (kend - kbeg + kG3K - 1) / kG3K;
    auto load = [&](int st) {
        if (st < nst) {
            float *b = sm3 + (st % kG3Stages) * kG3StageFloats;
            const int k0 = kbeg + st * kG3K;
#pragma unroll
            for (int i = 0; i < kG3WdFloats / 4 / kG3Threads; i++) {
                const int idx = tid + kG3Threads * i, kk = idx >> 5, q = idx & 31;   /* 32 quads per k */
                const bool ok = k0 + kk < kend;
                cp_async16_zfill((uint32_t)__cvta_generic_to_shared(b + kk * kG3Rows * 2 + 4 * q),
                                 ok ? (const void *)(Wd + ((size_t)(k0 + kk) * R + r0) * 2 + 4 * q) : (const void *)Wd,
                                 ok ? 16u : 0u);
            }
#pragma unroll
            for (int i = 0; i < kG3XFloats / 4 / kG3Threads; i++) {
                const int idx = tid + kG3Threads * i, kk = idx >> 4, q = idx & 15;   /* 16 quads per k */
                const int t = t0 + 4 * q;
                const int nb = k0 + kk < kend ? max(0, min(4, T - t)) * 4 : 0;
                cp_async16_zfill((uint32_t)__cvta_generic_to_shared(b + kG3WdFloats + kk * kG3Toks + 4 * q),
                                 nb ? (const void *)(xt + (size_t)(k0 + kk) * Tp + t) : (const void *)xt,
                                 (uint32_t)nb);
            }
            if (xr >= 0 && tid < kG3K / 4) {
                const int k = k0 + 4 * tid;
                const bool ok = k + 4 <= kend;
                cp_async16_zfill((uint32_t)__cvta_generic_to_shared(b + kG3WdFloats + kG3XFloats + 4 * tid),
                                 ok ? (const void *)(W + (size_t)xr * H + k) : (const void *)W, ok ? 16u : 0u);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");   /* empty groups keep the count uniform */
    };
    float2 acc[2][4][2][2], total[2][4][2][2];
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int bb = 0; bb < 2; bb++)
#pragma unroll
                for (int p = 0; p < 2; p++) total[a][i][bb][p] = acc[a][i][bb][p] = make_float2(0.0f, 0.0f);
    float ax = 0.0f, totx = 0.0f;
    for (int st = 0; st < kG3Stages - 1; st++) load(st);
    for (int st = 0; st < nst; st++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kG3Stages - 2) : "memory");
        __syncthreads();               /* stage st landed for every thread; stage st - 1's buffer is free */
        load(st + kG3Stages - 1);
        const float *b = sm3 + (st % kG3Stages) * kG3StageFloats;
        const int k0 = kbeg + st * kG3K, kn = min(kG3K, kend - k0);
        const float *wb = b + 8 * ty, *xb = b + kG3WdFloats + 4 * tx;
        auto step = [&](int kk) {
            float4 wv[2][2], xv[2];
#pragma unroll
            for (int a = 0; a < 2; a++) {
                wv[a][0] = *reinterpret_cast<const float4 *>(wb + kk * kG3Rows * 2 + 64 * a);
                wv[a][1] = *reinterpret_cast<const float4 *>(wb + kk * kG3Rows * 2 + 64 * a + 4);
            }
#pragma unroll
            for (int bb = 0; bb < 2; bb++) xv[bb] = *reinterpret_cast<const float4 *>(xb + kk * kG3Toks + 32 * bb);
#pragma unroll
            for (int a = 0; a < 2; a++)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float4 &w4 = wv[a][i >> 1];
                    const float2 w2 = (i & 1) ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y);
#pragma unroll
                    for (int bb = 0; bb < 2; bb++) {
                        acc[a][i][bb][0] = __ffma2_rn(w2, make_float2(xv[bb].x, xv[bb].y), acc[a][i][bb][0]);
                        acc[a][i][bb][1] = __ffma2_rn(w2, make_float2(xv[bb].z, xv[bb].w), acc[a][i][bb][1]);
                    }
                }
        };
        if (kn == kG3K) {
#pragma unroll
            for (int kk = 0; kk < kG3K; kk++) step(kk);
        } else {
#pragma unroll 1
            for (int kk = 0; kk < kn; kk++) step(kk);
        }
        if (xr >= 0) {   /* the gate row: its own chain, ascending k */
            const float *g = b + kG3WdFloats + kG3XFloats, *xg = b + kG3WdFloats + tid;
            for (int kk = 0; kk < kn; kk++) ax = __fmaf_rn(g[kk], xg[kk * kG3Toks], ax);
        }
        const bool chunk_end = ((k0 - kbeg + kG3K) % kChunk) == 0 || k0 + kG3K >= kend;
        if (chunk_end) {
            const int c = (k0 - kbeg) / kChunk + cbeg;
            if constexpr (kSplit) {   /* part[c][row][token] */
#pragma unroll
                for (int a = 0; a < 2; a++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int r = r0 + 32 * a + 4 * ty + i;
                        if (r >= Ep1 || r >= R) continue;
                        float *dst = part + ((size_t)c * Ep1 + r) * T;
#pragma unroll
                        for (int bb = 0; bb < 2; bb++)
#pragma unroll
                            for (int p = 0; p < 2; p++) {
                                const int t = t0 + 32 * bb + 4 * tx + 2 * p;
                                if (t < T) dst[t] = acc[a][i][bb][p].x;
                                if (t + 1 < T) dst[t + 1] = acc[a][i][bb][p].y;
                            }
                    }
                if (xr >= 0 && t0 + tid < T) part[((size_t)c * Ep1 + xr) * T + t0 + tid] = ax;
            } else {                  /* chunks added in order */
#pragma unroll
                for (int a = 0; a < 2; a++)
#pragma unroll
                    for (int i = 0; i < 4; i++)
#pragma unroll
                        for (int bb = 0; bb < 2; bb++)
#pragma unroll
                            for (int p = 0; p < 2; p++)
                                total[a][i][bb][p] = __fadd2_rn(total[a][i][bb][p], acc[a][i][bb][p]);
                totx = __fadd_rn(totx, ax);
            }
#pragma unroll
            for (int a = 0; a < 2; a++)
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int bb = 0; bb < 2; bb++)
#pragma unroll
                        for (int p = 0; p < 2; p++) acc[a][i][bb][p] = make_float2(0.0f, 0.0f);
            ax = 0.0f;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if constexpr (!kSplit) {
#pragma unroll
        for (int a = 0; a < 2; a++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = r0 + 32 * a + 4 * ty + i;
                if (r >= Ep1 || r >= R) continue;
                const float bv = bias && r < E ? bias[r] : 0.0f;
#pragma unroll
                for (int bb = 0; bb < 2; bb++)
#pragma unroll
                    for (int p = 0; p < 2; p++) {
                        const int t = t0 + 32 * bb + 4 * tx + 2 * p;
                        const float2 v = total[a][i][bb][p];
                        if (t < T) logits[(size_t)t * Ep1 + r] = bias && r < E ? __fadd_rn(v.x, bv) : v.x;
                        if (t + 1 < T) logits[(size_t)(t + 1) * Ep1 + r] = bias && r < E ? __fadd_rn(v.y, bv) : v.y;
                    }
            }
        if (xr >= 0 && t0 + tid < T)
            logits[(size_t)(t0 + tid) * Ep1 + xr] = bias && xr < E ? __fadd_rn(totx, bias[xr]) : totx;
    }
}

/* xt[k][t] = x[t][k] (row stride Tp), 32 x 32 tiles through shared memory. */
__global__ void router_transpose_x_kernel(const float *__restrict__ x, int T, int H, int Tp, float *__restrict__ xt) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.x * 32, tb = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const int t = tb + ty + i, k = k0 + tx;
        tile[ty + i][tx] = t < T && k < H ? x[(size_t)t * H + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const int k = k0 + ty + i, t = tb + tx;
        if (k < H && t < Tp) xt[(size_t)k * Tp + t] = tile[tx][ty + i];
    }
}

/* Wd[k][r][0] = Wd[k][r][1] = W[r][k] for the R rows of the paired-FMA router GEMM (zero past row E). */
__global__ void router_wd_fill_kernel(const float *__restrict__ W, int H, int E, int R, float *__restrict__ Wd) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)H * R) return;
    const int r = (int)(i % R), k = (int)(i / R);
    const float v = r <= E ? W[(size_t)r * H + k] : 0.0f;
    reinterpret_cast<float2 *>(Wd)[i] = make_float2(v, v);
}

/* logits[t][r] = (((0 + part[0][r][t]) + part[1][r][t]) + ...) + bias[r]: or_dot_f32's chunk order; one
 * thread per (r, t), consecutive threads consecutive tokens (coalesced reads of part). */
__global__ void router_sum2_kernel(const float *__restrict__ part, const float *__restrict__ bias, int nch, int T,
                                   int E, float *__restrict__ logits) {
    const int Ep1 = E + 1;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * Ep1) return;
    const int t = (int)(i % T), r = (int)(i / T);
    const size_t stride = (size_t)Ep1 * T;
    const float *p = part + (size_t)r * T + t;
    float tot = 0.0f;
    int c = 0;
    for (; c + 8 <= nch; c += 8) {   /* eight independent loads in flight, then the adds in chunk order */
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = p[(size_t)(c + j) * stride];
#pragma unroll
        for (int j = 0; j < 8; j++) tot = __fadd_rn(tot, v[j]);
    }
    for (; c < nch; c++) tot = __fadd_rn(tot, p[(size_t)c * stride]);
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

/* The same arithmetic for a compile-time code width and group size: the group's code words loaded up front, the
 * activations as float4, codes extracted with constant shifts; the two sums keep their sequential order. */
template <int BITS, int GS>
__global__ void router_qmat_exact_t_kernel(QeQDev m, int row_base, const float *__restrict__ x, int T, int H, int ld,
                                           float *__restrict__ logits) {
    constexpr int PER = 32 / BITS, WPG = GS * BITS / 32;
    constexpr uint32_t kMask = (1u << BITS) - 1u;
    const int lane = threadIdx.x & 31;
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row = (int)(wid % m.rows), t = (int)(wid / m.rows);
    if (t >= T) return;
    const int ng = m.cols / GS, wpr = m.cols * BITS / 32;
    const uint32_t *wp = m.w + (size_t)row * wpr;
    const float *xv = x + (size_t)t * H;
    float total = 0.0f;
    for (int g0 = 0; g0 < ng; g0 += 32) {
        const int g = g0 + lane;
        float tg = 0.0f;
        if (g < ng) {
            uint32_t w[WPG];
            const uint4 *gw4 = reinterpret_cast<const uint4 *>(wp + (size_t)g * WPG);
#pragma unroll
            for (int i = 0; i < WPG / 4; i++) {
                const uint4 u = __ldg(gw4 + i);
                w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
            }
            const float4 *x4 = reinterpret_cast<const float4 *>(xv + (size_t)g * GS);
            float gsum = 0.0f, sq = 0.0f;
#pragma unroll
            for (int c = 0; c < GS / 4; c++) {
                const float4 v = __ldg(x4 + c);
                const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int j = 4 * c + u;
                    gsum = __fadd_rn(gsum, xs[u]);
                    const float q = (float)((w[j / PER] >> ((j % PER) * BITS)) & kMask);
                    sq = __fadd_rn(sq, __fmul_rn(q, xs[u]));
                }
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

int qe_router_wd_rows(int E) { return (E + 1) % kG3Rows == 1 && E + 1 > kG3Rows ? E : (E + kG3Rows) / kG3Rows * kG3Rows; }

int qe_launch_router_wd_fill(const float *W, int H, int E, float *Wd, cudaStream_t s) {
    const int R = qe_router_wd_rows(E);
    const long long n = (long long)H * R;
    router_wd_fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(W, H, E, R, Wd);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_router_f32(const float *W, const float *bias, const float *x, int T, int H, int E, float *logits,
                         float *part, const float *Wd, float *xt, cudaStream_t s) {
    if (H > 32 * kMaxLaneChunks * kChunk) QE_FAIL("router: hidden %d too large", H);
    int launches = 1;
    if (T <= 16) {
        /* one warp (router row) per CTA: every SM streams router rows (4 per CTA left 83 of 148 SMs idle) */
        const int rows = E + 1, warps_per_block = 1;
        const int vec = H % 4 == 0 && ((uintptr_t)W | (uintptr_t)x) % 16 == 0;
        router_gemv_f32_kernel<<<(rows + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(
            W, bias, x, T, H, E, logits, vec);
    } else {
        if (H % 4) QE_FAIL("router: hidden %d must be a multiple of 4", H);
        const int nch = (H + kChunk - 1) / kChunk;
        if (Wd && xt && ((uintptr_t)W | (uintptr_t)Wd | (uintptr_t)xt) % 16 == 0) {
            /* paired-FMA GEMM on the handle's duplicated weights and the transposed batch */
            const int R = qe_router_wd_rows(E), xrow = R < E + 1 ? E : -1, Tp = (T + 3) & ~3;
            const int nrt = R / kG3Rows, ntt = (T + kG3Toks - 1) / kG3Toks, tiles = nrt * ntt;
            int dev = 0, sms = 148;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            router_transpose_x_kernel<<<dim3((H + 31) / 32, (Tp + 31) / 32), dim3(32, 8), 0, s>>>(x, T, H, Tp, xt);
            QE_CHECK(cudaGetLastError());
            launches = 2;
            if (tiles >= 2 * sms || !part) {
                router_gemm3_f32_kernel<false><<<dim3(nrt, ntt), kG3Threads, 0, s>>>(Wd, R, W, bias, xt, Tp, T, H, E,
                                                                                   nullptr, logits, nch, xrow);
            } else {
                /* about 12 CTAs per SM in all (6 resident): the chunks split over grid z */
                const long long want = 12LL * sms;
                const int cg = (int)std::max(1LL, ((long long)nch * tiles + want - 1) / want);
                router_gemm3_f32_kernel<true><<<dim3(nrt, ntt, (nch + cg - 1) / cg), kG3Threads, 0, s>>>(
                    Wd, R, W, bias, xt, Tp, T, H, E, part, nullptr, cg, xrow);
                QE_CHECK(cudaGetLastError());
                const long long n = (long long)T * (E + 1);
                router_sum2_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, bias, nch, T, E, logits);
                launches = 3;
            }
            QE_CHECK(cudaGetLastError());
            return launches;
        }
        /* 64n + 1 router rows: the last row tile's CTAs also compute the last row */
        const int xrow = (E + 1) % kGR2 == 1 && E + 1 > kGR2 ? E : -1;
        const int nrt = xrow >= 0 ? (E + 1) / kGR2 : (E + 1 + kGR2 - 1) / kGR2, ntt = (T + kGT2 - 1) / kGT2;
        const int tiles = nrt * ntt;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (((uintptr_t)W | (uintptr_t)x) % 16 == 0 && tiles >= 2 * sms) {
            /* enough tiles without splitting the inputs: every CTA adds its chunks itself */
            const size_t smem = sizeof(float) * 2 * (kWRows2 + kGT2) * kLds;
            dim3 grid(nrt, ntt);
            QE_CHECK(qe_set_smem((const void *)router_gemm2_f32_kernel<false>, smem));
            router_gemm2_f32_kernel<false><<<grid, kG2Threads, smem, s>>>(W, bias, x, T, H, E, nullptr, logits, nch,
                                                                          2, xrow);
        } else if (part && ((uintptr_t)W | (uintptr_t)x) % 16 == 0) {
            /* about 8 CTAs per SM in all: one chunk each (single-buffered, 6 CTAs resident per SM) for small
             * batches, more chunks per CTA (double-buffered) for larger ones */
            const long long want = 8LL * sms;
            const int cg = (int)std::max(1LL, ((long long)nch * tiles + want - 1) / want);
            const int nbuf = cg > 1 ? 2 : 1;
            const size_t smem = sizeof(float) * nbuf * (kWRows2 + kGT2) * kLds;
            dim3 grid(nrt, ntt, (nch + cg - 1) / cg);
            QE_CHECK(qe_set_smem((const void *)router_gemm2_f32_kernel<true>, smem));
            router_gemm2_f32_kernel<true><<<grid, kG2Threads, smem, s>>>(W, bias, x, T, H, E, part, nullptr, cg, nbuf,
                                                                         xrow);
            QE_CHECK(cudaGetLastError());
            const long long n = (long long)T * (E + 1);
            router_sum2_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, bias, nch, T, E, logits);
            launches = 2;
        } else if (part) {
            dim3 grid((E + 1 + kGR - 1) / kGR, (T + kGT - 1) / kGT, (nch + kCG - 1) / kCG);
            router_gemm_f32_kernel<true><<<grid, 128, 0, s>>>(W, bias, x, T, H, E, logits, part);
            QE_CHECK(cudaGetLastError());
            const long long n = (long long)T * (E + 1);
            router_sum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, bias, nch, T, E, logits);
            launches = 2;
        } else {
            dim3 grid((E + 1 + kGR - 1) / kGR, (T + kGT - 1) / kGT);
            router_gemm_f32_kernel<false><<<grid, 128, 0, s>>>(W, bias, x, T, H, E, logits, nullptr);
        }
    }
    QE_CHECK(cudaGetLastError());
    return launches;
}

/* One quantized router matrix's logits: the templated kernel for the usual code widths and group sizes (16-byte
 * aligned rows of codes and activations), the general one otherwise; the arithmetic is the same. */
static int launch_router_qmat_one(const QeQDev *m, int row_base, const float *x, int T, int H, int ld, float *logits,
                                  cudaStream_t s) {
    const long long warps = (long long)m->rows * T;
    const unsigned grid = (unsigned)((warps + 3) / 4);
    const bool aligned = H % 4 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)m->w % 16) == 0 &&
                         (m->cols * m->bits / 32) % 4 == 0;
    const int b = m->bits, gs = m->group_size;
    if (aligned && b == 4 && gs == 64) router_qmat_exact_t_kernel<4, 64><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else if (aligned && b == 8 && gs == 64) router_qmat_exact_t_kernel<8, 64><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else if (aligned && b == 4 && gs == 32) router_qmat_exact_t_kernel<4, 32><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else if (aligned && b == 8 && gs == 32) router_qmat_exact_t_kernel<8, 32><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else if (aligned && b == 4 && gs == 128) router_qmat_exact_t_kernel<4, 128><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else if (aligned && b == 8 && gs == 128) router_qmat_exact_t_kernel<8, 128><<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    else router_qmat_exact_kernel<<<grid, 128, 0, s>>>(*m, row_base, x, T, H, ld, logits);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_router_qmat(const QeQDev *router, const QeQDev *sh_router, const float *x, int T, int H, int E,
                          float *logits, cudaStream_t s) {
    if (launch_router_qmat_one(router, 0, x, T, H, E + 1, logits, s)) return -1;
    if (sh_router && launch_router_qmat_one(sh_router, E, x, T, H, E + 1, logits, s)) return -1;
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
