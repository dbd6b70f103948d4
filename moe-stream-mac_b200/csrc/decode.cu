/* decode.cu: the expert stage of a decode step (a handful of tokens) as CUDA-core GEMVs.
 *
 * Reference: engine/src/moe_layer.c:20-26 (mlp: gate, up, silu*up, down), :79-88 (combine in top-k order,
 * then the sigmoid-gated shared expert), engine/src/qmat.c:15-49 (per row, per group of 64:
 * scale*sum(q*x) + bias*sum(x)), engine/src/qgroup.c (code j of a group at bit (j % (32/bits))*bits of word
 * j / (32/bits), LSB first).
 *
 * At one token per expert there is nothing to reuse: each selected expert's packed codes are read once, and
 * the work is the HBM stream. Two kernels:
 *   decode_gateup_kernel      one CTA per (token-slot pair, block of rows): h = silu(gate.x) * (up.x)
 *   decode_down_combine_kernel one CTA per (token, block of output rows): y_j = down_j . h_j for the k routed
 *                             slots and the shared expert, out = sum_j score_j y_j (slot order) + sg y_shared
 * A row is read by a sub-warp of SW lanes with 16-byte loads, NL per lane, every load of the warp's R rows
 * issued before any arithmetic. Lane l of load i holds bytes [(i*SW + l)*16, +16) of the row: 32 codes
 * (4-bit) or 16 (8-bit), so 2 or 4 consecutive lanes hold one group of 64. Each lane forms its codes' fp32
 * dot with x (sequential), the group's lanes add their parts, the group's first lane forms
 * scale*sum_q + bias*sum_x (qmat.c:43) and the row total is a shuffle tree over the sub-warp. fp32
 * throughout; the order differs from the reference's (tolerance 1e-5 rel-L2).
 */
#include "qe_common.cuh"
#include "qe_kernels.h"

namespace {

constexpr int kThreads = 256;   /* 8 warps */
constexpr int kGS = 64;

/* Code q as the float 1 + q/16 (4-bit) or 1 + q/256 (8-bit): the code's bits are the top mantissa bits, one
 * shift and one logic op. Sum_i (1 + q_i/2^b) x_i - Sum_i x_i = 2^-b Sum_i q_i x_i, so a lane forms its dot
 * with paired fp32 FMAs and subtracts its chunk's x sum; the cancellation costs ~2 bits of the 24 (the terms
 * are within a factor ~2 of the result). */
template <int BITS, int I>
__device__ __forceinline__ float code_v(uint32_t w) {
    constexpr int kTop = 23 - BITS;                 /* mantissa position of the code's lowest bit */
    constexpr int kSh = kTop - BITS * I;            /* left shift bringing code I there */
    constexpr uint32_t kMask = ((1u << BITS) - 1u) << kTop;
    const uint32_t s = kSh >= 0 ? (w << (kSh >= 0 ? kSh : 0)) : (w >> (kSh < 0 ? -kSh : 0));
    return __uint_as_float((s & kMask) | 0x3F800000u);
}

/* 2^-b * (dot of one lane's 16 code bytes with its x values), given the lane's x sum */
template <int BITS>
__device__ __forceinline__ float lane_dot(const uint4 w, const float *xs, float xsum) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        if constexpr (BITS == 4) {
            a = __ffma2_rn(make_float2(code_v<4, 0>(ws[q]), code_v<4, 1>(ws[q])), make_float2(xs[q * 8], xs[q * 8 + 1]), a);
            a = __ffma2_rn(make_float2(code_v<4, 2>(ws[q]), code_v<4, 3>(ws[q])), make_float2(xs[q * 8 + 2], xs[q * 8 + 3]), a);
            a = __ffma2_rn(make_float2(code_v<4, 4>(ws[q]), code_v<4, 5>(ws[q])), make_float2(xs[q * 8 + 4], xs[q * 8 + 5]), a);
            a = __ffma2_rn(make_float2(code_v<4, 6>(ws[q]), code_v<4, 7>(ws[q])), make_float2(xs[q * 8 + 6], xs[q * 8 + 7]), a);
        } else {
            a = __ffma2_rn(make_float2(code_v<8, 0>(ws[q]), code_v<8, 1>(ws[q])), make_float2(xs[q * 4], xs[q * 4 + 1]), a);
            a = __ffma2_rn(make_float2(code_v<8, 2>(ws[q]), code_v<8, 3>(ws[q])), make_float2(xs[q * 4 + 2], xs[q * 4 + 3]), a);
        }
    }
    return __fsub_rn(__fadd_rn(a.x, a.y), xsum);
}

/* Shared-memory vectors are stored with their 16-byte pieces swizzled within each lane chunk (Q pieces):
 * piece q of chunk c sits at q ^ (c % Q), so the 32 lanes of a warp, reading piece q of consecutive chunks,
 * hit distinct banks. */
template <int Q>
__device__ __forceinline__ int swz(int c, int q) { return q ^ (c & (Q - 1)); }

/* The code words of R rows (bytes per row = NL*SW*16) for one sub-warp lane, and the scale and bias of each
 * lane-load's group (bf16 pairs, scale in the low half), all requested together. */
template <int BITS, int SW, int NL, int R>
__device__ __forceinline__ void load_rows(const uint8_t *const (&rows)[R], const uint16_t *const (&sc)[R],
                                          const uint16_t *const (&bi)[R], size_t gstride, int sl, uint4 (&w)[R][NL],
                                          uint32_t (&sb)[R][NL]) {
    constexpr int LPG = kGS / (128 / BITS);
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int i = 0; i < NL; i++) {
            w[r][i] = __ldg(reinterpret_cast<const uint4 *>(rows[r]) + i * SW + sl);
            const size_t g = (size_t)((i * SW + sl) / LPG) * gstride;
            sb[r][i] = (uint32_t)__ldg(sc[r] + g) | ((uint32_t)__ldg(bi[r] + g) << 16);
        }
}

/* Row r's loaded codes dotted with x[r] (shared memory, fp32) by a sub-warp of SW lanes; cs[r]: x[r]'s sums
 * per lane chunk (128/BITS elements), gsum[r]: per group of 64; sc/bi: scale/bias of (row, group g) at
 * sc[g * gstride]. Returns the row totals in every lane of the sub-warp. */
template <int BITS, int SW, int NL, int R, bool SAMEX>
__device__ __forceinline__ void dot_rows(const uint4 (&w)[R][NL], const uint32_t (&sb)[R][NL],
                                         const float *const (&x)[R], const float *const (&cs)[R],
                                         const float *const (&gsum)[R], int sl, float (&tot)[R]) {
    constexpr int CPL = 128 / BITS;   /* codes per lane-load */
    constexpr int LPG = kGS / CPL;    /* lanes per group */
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < NL; i++) {
        const int lp = i * SW + sl;          /* lane-load position in the row */
        const int g = lp / LPG;
        float xs[CPL];
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (r == 0 || !SAMEX) {   /* rows sharing one vector (gate/up) read it once */
                const float4 *x4 = reinterpret_cast<const float4 *>(x[r]) + lp * (CPL / 4);
#pragma unroll
                for (int q = 0; q < CPL / 4; q++) {
                    const float4 v = x4[swz<CPL / 4>(lp, q)];
                    xs[4 * q] = v.x; xs[4 * q + 1] = v.y; xs[4 * q + 2] = v.z; xs[4 * q + 3] = v.w;
                }
            }
            float part = lane_dot<BITS>(w[r][i], xs, cs[r][lp]);
#pragma unroll
            for (int o = 1; o < LPG; o <<= 1) part = __fadd_rn(part, __shfl_xor_sync(QE_FULL, part, o));
            if (lp % LPG == 0) {
                const float sq = __fmul_rn(part, (float)(1 << BITS));   /* exact: a power of two */
                const float s = __uint_as_float(sb[r][i] << 16), b = __uint_as_float(sb[r][i] & 0xFFFF0000u);
                acc[r] = __fadd_rn(acc[r], __fmaf_rn(s, sq, __fmul_rn(b, gsum[r][g])));
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
        float v = acc[r];
#pragma unroll
        for (int o = 1; o < SW; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(QE_FULL, v, o));
        tot[r] = v;
    }
}

/* n vectors of K floats into shared memory (vs[j*ldv + c]) with their sums per chunk of `chunk` elements
 * (cs[j*(ldv/chunk) + c]) and per group of 64 (gs[j*(ldv/64) + g]), all sequential in element order.
 * src(j) gives vector j's global address. */
template <int CHUNK, typename Src>
__device__ void stage_vecs(Src src, int n, int K, int ldv, float *vs, float *cs, float *gs) {
    constexpr int Q = CHUNK / 4;
    for (int i = threadIdx.x; i < n * ldv; i += blockDim.x) {
        const int j = i / ldv, c = i % ldv;
        const int ch = c / CHUNK, q = (c % CHUNK) / 4;
        vs[(size_t)j * ldv + ch * CHUNK + swz<Q>(ch, q) * 4 + (c & 3)] = c < K ? src(j)[c] : 0.0f;
    }
    __syncthreads();
    const int nc = ldv / CHUNK;
    for (int i = threadIdx.x; i < n * nc; i += blockDim.x) {
        const int ch = i % nc;
        const float *v = vs + (size_t)(i / nc) * ldv + (size_t)ch * CHUNK;
        float s = 0.0f;
        for (int c = 0; c < CHUNK; c++) s = __fadd_rn(s, v[swz<Q>(ch, c / 4) * 4 + (c & 3)]);
        cs[i] = s;
    }
    __syncthreads();
    const int ng = ldv / kGS, per = kGS / CHUNK;
    for (int i = threadIdx.x; i < n * ng; i += blockDim.x) {
        const float *c = cs + (size_t)(i / ng) * nc + (size_t)(i % ng) * per;
        float s = 0.0f;
        for (int q = 0; q < per; q++) s = __fadd_rn(s, c[q]);
        gs[i] = s;
    }
    __syncthreads();
}

/* The quantized matrix (routed expert e, or the shared one) as row pointers: codes of row `row`, and the
 * scale/bias of (row, group 0) with the stride between groups (expert tensors keep [n][groups][rows]). */
struct QRow {
    const uint8_t *codes;
    const uint16_t *sc, *bi;
    size_t gstride;
};
__device__ __forceinline__ QRow qrow(const QeQDev &m, int e, int row) {
    const int ng = m.cols / kGS;
    const size_t bpr = (size_t)m.cols * m.bits / 8;
    QRow q;
    q.codes = reinterpret_cast<const uint8_t *>(m.w) + ((size_t)e * m.rows + row) * bpr;
    if (m.scale_t) {
        const size_t o = (size_t)e * ng * m.rows + row;
        q.sc = m.scales + o;
        q.bi = m.biases + o;
        q.gstride = m.rows;
    } else {
        const size_t o = ((size_t)e * m.rows + row) * ng;
        q.sc = m.scales + o;
        q.bi = m.biases + o;
        q.gstride = 1;
    }
    return q;
}

/* Rows per warp pass: each sub-warp takes R rows at once. */
constexpr int kR = 2;

template <int BITS, int SW, int NL>
__global__ void __launch_bounds__(kThreads) decode_gateup_kernel(QeExpertArgs a, const float *__restrict__ x,
                                                                 const int32_t *__restrict__ idx, int k,
                                                                 float *__restrict__ h3, int ldh, int rows_per_cta) {
    extern __shared__ __align__(16) float smem[];
    const int p = blockIdx.x;                 /* pair t*(k+1) + j */
    const int t = p / (k + 1), j = p % (k + 1);
    const bool shared = j == k;
    const int e = shared ? 0 : idx[(size_t)t * k + j];
    const QeQDev &G = shared ? a.sh_gate : a.gate, &U = shared ? a.sh_up : a.up;
    const int rows = G.rows, K = G.cols;
    constexpr int CPL = 128 / BITS;
    float *xs = smem, *cs = smem + K, *gsum = cs + K / CPL;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int SUBS = 32 / SW;
    const int sub = lane / SW, sl = lane % SW;
    const int r0 = blockIdx.y * rows_per_cta;
    const int r1 = min(rows, r0 + rows_per_cta);
    /* sub-warp (warp, sub) owns rows rb .. rb+kR-1 of each pass; the loop bound is the warp's first row so
     * every lane of a warp runs the same iterations (the shuffles need all 32); past r1, rows are clamped and
     * their results dropped. The first pass's code words are requested before x is staged. */
    bool staged = false;
    for (int rw = r0 + warp * SUBS * kR; ; rw += (kThreads / 32) * SUBS * kR) {
        const bool work = rw < r1;
        const int rb = rw + sub * kR;
        const uint8_t *rp[2 * kR];
        const uint16_t *sp[2 * kR], *bp[2 * kR];
        size_t gstride = 0;
#pragma unroll
        for (int q = 0; q < kR; q++) {
            const int row = max(r0, min(rb + q, r1 - 1));
            const QRow g = qrow(G, e, row), u = qrow(U, e, row);
            rp[2 * q] = g.codes; sp[2 * q] = g.sc; bp[2 * q] = g.bi;
            rp[2 * q + 1] = u.codes; sp[2 * q + 1] = u.sc; bp[2 * q + 1] = u.bi;
            gstride = g.gstride;
        }
        uint4 w[2 * kR][NL];
        uint32_t sb[2 * kR][NL];
        if (work) load_rows<BITS, SW, NL, 2 * kR>(rp, sp, bp, gstride, sl, w, sb);
        if (!staged) {   /* every thread reaches this once, on its first iteration */
            stage_vecs<CPL>([&](int) { return x + (size_t)t * K; }, 1, K, K, xs, cs, gsum);
            staged = true;
        }
        if (!work) break;
        float tot[2 * kR];
        const float *xr[2 * kR], *cr[2 * kR], *gr[2 * kR];
#pragma unroll
        for (int q = 0; q < 2 * kR; q++) {
            xr[q] = xs;
            cr[q] = cs;
            gr[q] = gsum;
        }
        dot_rows<BITS, SW, NL, 2 * kR, true>(w, sb, xr, cr, gr, sl, tot);
        if (sl == 0)
#pragma unroll
            for (int q = 0; q < kR; q++)
                if (rb + q < r1) h3[(size_t)p * ldh + rb + q] = qe_silu_mul(tot[2 * q], tot[2 * q + 1]);
    }
}

template <int BITS, int SW, int NL>
__global__ void __launch_bounds__(kThreads) decode_down_combine_kernel(QeExpertArgs a, const float *__restrict__ h3,
                                                                       int ldh, const int32_t *__restrict__ idx,
                                                                       const float *__restrict__ score,
                                                                       const float *__restrict__ logits, int ld_logits,
                                                                       int E, int k, float *__restrict__ out,
                                                                       int rows_per_cta) {
    extern __shared__ __align__(16) float smem[];
    constexpr int CPL = 128 / BITS;
    const int t = blockIdx.x;
    const int kp1 = k + 1;
    const int K = a.down.cols, H = a.hidden;   /* the shared expert's down has the same K (checked at launch) */
    /* the token's k+1 activation vectors, their chunk sums and group sums */
    float *hs = smem, *cs = hs + (size_t)kp1 * K, *gsum = cs + (size_t)kp1 * (K / CPL);
    const float sg = qe_sigmoid(logits[(size_t)t * ld_logits + E]);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int SUBS = 32 / SW;
    const int sub = lane / SW, sl = lane % SW;
    const int r0 = blockIdx.y * rows_per_cta, r1 = min(H, r0 + rows_per_cta);
    /* a sub-warp takes one output row at a time and its k+1 slots (routed experts, then the shared one) in
     * passes of kRD, all loads of a pass in flight together; the combine runs in slot order (moe_layer.c:79-88).
     * The loop bound is warp-uniform (shuffles need all lanes); clamped rows are dropped. The first pass's code
     * words are requested before the activations are staged. */
    /* slots per pass: all 9 of a top-8 block when a row is one load per lane, fewer for longer rows (about 10
     * loads in flight per lane) */
    constexpr int kRD = NL <= 1 ? 9 : NL == 2 ? 5 : NL <= 4 ? 3 : 1;
    bool staged = false;
    for (int rw = r0 + warp * SUBS; ; rw += (kThreads / 32) * SUBS) {
        const bool work = rw < r1;
        const bool live = rw + sub < r1;
        const int row = live ? rw + sub : r1 - 1;
        float y[17];
        for (int j0 = 0; j0 < kp1; j0 += kRD) {
            const uint8_t *rp[kRD];
            const uint16_t *sp[kRD], *bp[kRD];
            const float *xr[kRD], *cr[kRD], *gr[kRD];
            size_t gstride = 0;
#pragma unroll
            for (int q = 0; q < kRD; q++) {
                const int j = min(j0 + q, kp1 - 1);
                const QRow d = j == k ? qrow(a.sh_down, 0, row) : qrow(a.down, idx[(size_t)t * k + j], row);
                rp[q] = d.codes; sp[q] = d.sc; bp[q] = d.bi;
                gstride = d.gstride;   /* the same for routed and shared down (equal shapes) */
                xr[q] = hs + (size_t)j * K;
                cr[q] = cs + (size_t)j * (K / CPL);
                gr[q] = gsum + (size_t)j * (K / kGS);
            }
            uint4 w[kRD][NL];
            uint32_t sb[kRD][NL];
            if (work) load_rows<BITS, SW, NL, kRD>(rp, sp, bp, gstride, sl, w, sb);
            if (!staged) {   /* every thread reaches this once, in its first pass */
                stage_vecs<CPL>([&](int j) { return h3 + ((size_t)t * kp1 + j) * ldh; }, kp1, K, K, hs, cs, gsum);
                staged = true;
            }
            if (!work) break;
            float tot[kRD];
            dot_rows<BITS, SW, NL, kRD, false>(w, sb, xr, cr, gr, sl, tot);
#pragma unroll
            for (int q = 0; q < kRD; q++)
                if (j0 + q < kp1) y[j0 + q] = tot[q];
        }
        if (!work) break;
        if (sl == 0 && live) {
            float o = 0.0f;
            for (int j = 0; j < k; j++) o = __fadd_rn(o, __fmul_rn(score[(size_t)t * k + j], y[j]));
            o = __fadd_rn(o, __fmul_rn(sg, y[k]));
            out[(size_t)t * H + row] = o;
        }
    }
}

/* (SW, NL) for a row of `bytes` bytes: whole warps (32 lanes) when the row has at least 512 bytes. */
bool shape_of(int bytes, int &sw, int &nl) {
    if (bytes % 16) return false;
    const int loads = bytes / 16;
    if (loads >= 32) {
        if (loads % 32) return false;
        sw = 32;
        nl = loads / 32;
    } else {
        if (loads != 8 && loads != 16) return false;
        sw = loads;
        nl = 1;
    }
    return nl == 1 || nl == 2 || nl == 3 || nl == 4 || nl == 6 || nl == 8;
}

template <int BITS, int SW, int NL>
int launch_gateup_t(const QeExpertArgs *a, const float *x, const int32_t *idx, int T, float *h3, int ldh,
                    cudaStream_t s) {
    const int rows = a->inter, K = a->hidden;
    const int rpc = 16;
    dim3 grid(T * (a->k + 1), (rows + rpc - 1) / rpc);
    const size_t smem = sizeof(float) * ((size_t)K + K / (128 / BITS) + K / kGS);
    decode_gateup_kernel<BITS, SW, NL><<<grid, kThreads, smem, s>>>(*a, x, idx, a->k, h3, ldh, rpc);
    QE_CHECK(cudaGetLastError());
    return 0;
}

template <int BITS, int SW, int NL>
int launch_down_t(const QeExpertArgs *a, const float *h3, int ldh, const int32_t *idx, const float *score,
                  const float *logits, int ld_logits, int T, float *out, cudaStream_t s) {
    const int rpc = 16;
    const int K = a->inter;
    if (a->sh_inter != K) QE_FAIL("decode down: shared expert width %d != %d", a->sh_inter, K);
    dim3 grid(T, (a->hidden + rpc - 1) / rpc);
    const size_t smem = sizeof(float) * (size_t)(a->k + 1) * ((size_t)K + K / (128 / BITS) + K / kGS);
    if (smem > 200 * 1024) QE_FAIL("decode down: %zu B of shared memory", smem);
    auto kern = decode_down_combine_kernel<BITS, SW, NL>;
    QE_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kThreads, smem, s>>>(*a, h3, ldh, idx, score, logits, ld_logits, a->E, a->k, out, rpc);
    QE_CHECK(cudaGetLastError());
    return 0;
}

#define QE_SHAPES(F, BITS, ...)                                                       \
    if (sw == 8 && nl == 1) return F<BITS, 8, 1>(__VA_ARGS__);                         \
    if (sw == 16 && nl == 1) return F<BITS, 16, 1>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 1) return F<BITS, 32, 1>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 2) return F<BITS, 32, 2>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 3) return F<BITS, 32, 3>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 4) return F<BITS, 32, 4>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 6) return F<BITS, 32, 6>(__VA_ARGS__);                       \
    if (sw == 32 && nl == 8) return F<BITS, 32, 8>(__VA_ARGS__);

}  // namespace

/* Whether the decode GEMVs cover this block: group size 64, rows of gate/up and of down of a supported byte
 * length, and the shared expert's down rows of the same length as the routed ones. */
bool qe_decode_supported(const QeExpertArgs *a) {
    const int bits = a->gate.bits;
    if (a->gate.group_size != kGS || (bits != 4 && bits != 8)) return false;
    if (a->inter != a->sh_inter) return false;
    int sw, nl;
    return shape_of(a->hidden * bits / 8, sw, nl) && shape_of(a->inter * bits / 8, sw, nl);
}

int qe_launch_decode_gateup(const QeExpertArgs *a, const float *x, const int32_t *idx, int T, float *h3, int ldh,
                            cudaStream_t s) {
    int sw = 0, nl = 0;
    if (!shape_of(a->hidden * a->gate.bits / 8, sw, nl)) QE_FAIL("decode gate/up: unsupported hidden %d", a->hidden);
    if (a->gate.bits == 4) {
        QE_SHAPES(launch_gateup_t, 4, a, x, idx, T, h3, ldh, s)
    } else {
        QE_SHAPES(launch_gateup_t, 8, a, x, idx, T, h3, ldh, s)
    }
    QE_FAIL("decode gate/up: no kernel for sw=%d nl=%d", sw, nl);
}

int qe_launch_decode_down_combine(const QeExpertArgs *a, const float *h3, int ldh, const int32_t *idx,
                                  const float *score, const float *logits, int ld_logits, int T, float *out,
                                  cudaStream_t s) {
    int sw = 0, nl = 0;
    if (!shape_of(a->inter * a->gate.bits / 8, sw, nl)) QE_FAIL("decode down: unsupported inter %d", a->inter);
    if (a->gate.bits == 4) {
        QE_SHAPES(launch_down_t, 4, a, h3, ldh, idx, score, logits, ld_logits, T, out, s)
    } else {
        QE_SHAPES(launch_down_t, 8, a, h3, ldh, idx, score, logits, ld_logits, T, out, s)
    }
    QE_FAIL("decode down: no kernel for sw=%d nl=%d", sw, nl);
}
