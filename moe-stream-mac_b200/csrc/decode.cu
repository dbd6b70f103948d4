/* decode.cu: the expert stage of a decode step (a handful of tokens) as CUDA-core GEMVs.
 *
 * Reference: engine/src/moe_layer.c:20-26 (mlp: gate, up, silu*up, down), :79-88 (combine in top-k order,
 * then the sigmoid-gated shared expert), engine/src/qmat.c:15-49 (per row, per group of 64:
 * scale*sum(q*x) + bias*sum(x)), engine/src/qgroup.c (code j of a group at bit (j % (32/bits))*bits of word
 * j / (32/bits), LSB first).
 *
 * At one token per expert nothing is reused: each selected expert's packed codes are read once, and the work
 * is the HBM stream. Two kernels, one or two lanes per weight row (every lane of a warp reads the same
 * activation element, a shared-memory broadcast):
 *   decode_gateup_kernel       CTA = (token-slot pair, 32 rows); warps 0-7 stream the gate rows, 8-15 the up
 *                              rows, each warp one eighth of K; parts summed in order, h = silu(g) * u
 *   decode_down_combine_kernel CTA = (token, 16 output rows); warp j streams slot j's down rows (k routed
 *                              experts, then the shared one), two lanes per row (each half of the row, the two
 *                              parts added in order); out = sum_j score_j y_j (slot order) + sg y_shared
 * A lane streams its row in 128-byte chunks (8 x 16-byte loads) through a 2-deep register ring, the chunk's
 * group scales and biases with it; the first loads are issued before the activations are staged. A code q is
 * formed as the float 1 + q/2^b (one shift, one logic op), dotted with x by paired fp32 FMAs, and the group's
 * x sum is subtracted: sum_i (1 + q_i/2^b) x_i - sum_i x_i = 2^-b sum_i q_i x_i (the cancellation costs about
 * 2 of the 24 bits). Then scale * sum_q + bias * sum_x per group (qmat.c:43), groups in order. fp32 throughout;
 * the order differs from the reference's (tolerance 1e-5 rel-L2).
 */
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "qe_common.cuh"
#include "qe_kernels.h"
#include "route_dev.cuh"
#include "gemv_dev.cuh"

namespace {

constexpr int kGS = 64;
constexpr int kFusedMaxTokens = 4;   /* tokens of a fused decode step (kDecodeMaxTokens in qe_moe.cu) */
#define QE_DECODE_WAIT_NS 2000000000ull

__device__ __forceinline__ uint64_t decode_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* 2^-b * sum_q q*x over one 16-byte word group (32 or 16 codes) against x (shared memory, broadcast) */
template <int BITS>
__device__ __forceinline__ float2 word_dot(const uint4 w, const float *x, float2 a) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        if constexpr (BITS == 4) {
            const float4 xa = x4[2 * q], xb = x4[2 * q + 1];
            a = __ffma2_rn(make_float2(code_v<4, 0>(ws[q]), code_v<4, 1>(ws[q])), make_float2(xa.x, xa.y), a);
            a = __ffma2_rn(make_float2(code_v<4, 2>(ws[q]), code_v<4, 3>(ws[q])), make_float2(xa.z, xa.w), a);
            a = __ffma2_rn(make_float2(code_v<4, 4>(ws[q]), code_v<4, 5>(ws[q])), make_float2(xb.x, xb.y), a);
            a = __ffma2_rn(make_float2(code_v<4, 6>(ws[q]), code_v<4, 7>(ws[q])), make_float2(xb.z, xb.w), a);
        } else {
            const float4 xa = x4[q];
            a = __ffma2_rn(make_float2(code_v<8, 0>(ws[q]), code_v<8, 1>(ws[q])), make_float2(xa.x, xa.y), a);
            a = __ffma2_rn(make_float2(code_v<8, 2>(ws[q]), code_v<8, 3>(ws[q])), make_float2(xa.z, xa.w), a);
        }
    }
    return a;
}

constexpr int kChunk = 128;            /* bytes a lane loads per ring slot */
constexpr int kU4 = kChunk / 16;

/* One lane streaming chunks [c0, c1) of its row: codes (8 x 16 B per chunk) and the chunk's groups' scales and
 * biases (bf16 pairs) through a 2-deep ring. */
template <int BITS>
struct RowStream {
    static constexpr int GB = 64 * BITS / 8;        /* bytes per group of 64 codes */
    static constexpr int GPC = kChunk / GB;         /* groups per chunk: 4 (4-bit) or 2 (8-bit) */
    const uint8_t *row;
    const uint16_t *sc, *bi;
    size_t gstride;
    int c0, c1;
    uint4 w[2][kU4];
    uint32_t sb[2][GPC];

    __device__ __forceinline__ void load(int slot, int c) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + (size_t)c * kChunk);
#pragma unroll
        for (int i = 0; i < kU4; i++) w[slot][i] = __ldg(p + i);
#pragma unroll
        for (int gi = 0; gi < GPC; gi++) {
            const size_t g = (size_t)(c * GPC + gi) * gstride;
            sb[slot][gi] = (uint32_t)__ldg(sc + g) | ((uint32_t)__ldg(bi + g) << 16);
        }
    }
    __device__ __forceinline__ void start() {
        if (c0 < c1) load(0, c0);
        if (c0 + 1 < c1) load(1, c0 + 1);
    }
    /* sum over the groups of the chunk in slot `slot`: scale*sum_q + bias*sum_x, added to acc in group order */
    __device__ __forceinline__ float chunk(int slot, int c, const float *x, const float *gsum, float acc) const {
#pragma unroll
        for (int gi = 0; gi < GPC; gi++) {
            const int g = c * GPC + gi;
            float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < GB / 16; i++)
                a = word_dot<BITS>(w[slot][gi * (GB / 16) + i], x + g * 64 + i * (128 / BITS), a);
            const float sq = __fmul_rn(__fsub_rn(__fadd_rn(a.x, a.y), gsum[g]), (float)(1 << BITS));
            const float s = __uint_as_float(sb[slot][gi] << 16), b = __uint_as_float(sb[slot][gi] & 0xFFFF0000u);
            acc = __fadd_rn(acc, __fmaf_rn(s, sq, __fmul_rn(b, gsum[g])));
        }
        return acc;
    }
    __device__ __forceinline__ float finish(const float *x, const float *gsum) {
        float acc = 0.0f;
        for (int c = c0; c < c1; c += 2) {
            acc = chunk(0, c, x, gsum, acc);
            if (c + 2 < c1) load(0, c + 2);
            if (c + 1 < c1) {
                acc = chunk(1, c + 1, x, gsum, acc);
                if (c + 3 < c1) load(1, c + 3);
            }
        }
        return acc;
    }
};

/* n vectors of K floats into shared memory (vs[j*K + c]) and their sums per group of 64 (gs[j*(K/64) + g]):
 * 16-byte copies (K a multiple of 4, rows 16-byte aligned), then one warp per group, a fixed shuffle tree.
 * src(j) gives vector j's global address. */
template <typename Src>
__device__ void stage_vecs(Src src, int n, int K, float *vs, float *gs) {
    const int k4 = K >> 2;
    int j = 0, c = threadIdx.x;   /* element c of vector j, advanced without divisions */
    while (true) {
        while (c >= k4 && j < n) {
            c -= k4;
            j++;
        }
        if (j >= n) break;
        reinterpret_cast<float4 *>(vs)[(size_t)j * k4 + c] = __ldg(reinterpret_cast<const float4 *>(src(j)) + c);
        c += blockDim.x;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5, ng = K / kGS;
    for (int i = warp; i < n * ng; i += nw) {
        const float *v = vs + (size_t)(i / ng) * K + (size_t)(i % ng) * kGS;
        float s = __fadd_rn(v[2 * lane], v[2 * lane + 1]);
#pragma unroll
        for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(QE_FULL, s, o));
        if (lane == 0) gs[i] = s;
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

constexpr int kParts = 8;   /* K parts per matrix in the gate/up kernel */
/* Down kernel: two lanes per output row, each streaming half of the row's chunks, 16 rows per CTA: twice the
 * CTAs of one lane per row (128 for hidden 2048 at one token, against 64), 11% faster decode steps on C1 and
 * the same on C3 (B200); four lanes per row were slower at 8 bits. */
constexpr int kDownLanesPerRow = 2, kDownRows = 32 / kDownLanesPerRow;
constexpr int kGuThreads = 2 * kParts * 32;

/* Gate/up + SwiGLU of one (token-slot pair p, 32-row block at r0): warps 0-7 stream the gate rows, 8-15 the up
 * rows, each warp one eighth of K; parts summed in order, h = silu(g) * u -> h3[p][r0 + lane]. idx: the top-k
 * ids [T][k] (global or shared memory). All 512 threads of the CTA call it; xs: hidden + hidden/64 floats of
 * shared memory. */
template <int BITS>
__device__ __forceinline__ void gateup_unit(const QeExpertArgs &a, const float *__restrict__ x, const int32_t *idx,
                                            int k, float *__restrict__ h3, int ldh, int p, int r0, float *xs,
                                            float (*part_sum)[32]) {
    const int t = p / (k + 1), j = p % (k + 1);
    const bool shared = j == k;
    const int e = shared ? 0 : idx[t * k + j];
    const QeQDev &G = shared ? a.sh_gate : a.gate, &U = shared ? a.sh_up : a.up;
    const int rows = G.rows, K = G.cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = warp / kParts, part = warp % kParts;
    const int row = min(r0 + lane, rows - 1);
    const int nch = K * BITS / 8 / kChunk;
    const QRow q = qrow(m ? U : G, e, row);
    RowStream<BITS> st;
    st.row = q.codes; st.sc = q.sc; st.bi = q.bi; st.gstride = q.gstride;
    st.c0 = part * nch / kParts;
    st.c1 = (part + 1) * nch / kParts;
    st.start();                               /* codes in flight while x is staged */
    float *gsum = xs + K;
    stage_vecs([&](int) { return x + (size_t)t * K; }, 1, K, xs, gsum);
    part_sum[warp][lane] = st.finish(xs, gsum);
    __syncthreads();
    if (warp == 0 && r0 + lane < rows) {
        float g = 0.0f, u = 0.0f;
        for (int i = 0; i < kParts; i++) {
            g = __fadd_rn(g, part_sum[i][lane]);
            u = __fadd_rn(u, part_sum[kParts + i][lane]);
        }
        h3[(size_t)p * ldh + r0 + lane] = qe_silu_mul(g, u);
    }
}

template <int BITS>
__global__ void __launch_bounds__(kGuThreads) decode_gateup_kernel(QeExpertArgs a, const float *__restrict__ x,
                                                                   const int32_t *__restrict__ idx, int k,
                                                                   float *__restrict__ h3, int ldh) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float part_sum[2 * kParts][32];
    gateup_unit<BITS>(a, x, idx, k, h3, ldh, blockIdx.x, blockIdx.y * 32, smem, part_sum);
}

/* Down projection of token t's k+1 slots for the 32 output rows at r0, combined in slot order: warp j < k+1
 * streams slot j's down rows (k routed experts, then the shared one). begin() requests the codes; end() stages
 * the token's k+1 activation vectors (shared memory hs: (k+1) * (K + K/64) floats), finishes the dots and
 * writes out = sum_j score_j y_j (slot order) + sigmoid(gate logit) y_shared (moe_layer.c:79-88). */
template <int BITS, int LPR = 1>
struct DownUnit {
    RowStream<BITS> st;
    int t, r0;
    __device__ __forceinline__ void begin(const QeExpertArgs &a, const int32_t *idx, int k, int t_, int r0_) {
        t = t_;
        r0 = r0_;
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int H = a.hidden, row = min(r0 + lane / LPR, H - 1), part = lane % LPR;
        st.c0 = 0;
        st.c1 = 0;
        if (warp > k) return;
        const QRow q = warp == k ? qrow(a.sh_down, 0, row) : qrow(a.down, idx[t * k + warp], row);
        st.row = q.codes; st.sc = q.sc; st.bi = q.bi; st.gstride = q.gstride;
        const int nch = a.down.cols * BITS / 8 / kChunk;   /* LPR lanes share a row: chunk ranges split */
        st.c0 = part * nch / LPR;
        st.c1 = (part + 1) * nch / LPR;
        st.start();
    }
    __device__ __forceinline__ void end(const QeExpertArgs &a, const float *__restrict__ h3, int ldh, int k,
                                        const float *score, const float *__restrict__ logits, int ld_logits,
                                        float *__restrict__ out, float *hs, float (*ys)[32]) {
        const int kp1 = k + 1, K = a.down.cols, H = a.hidden;
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        float *gsum = hs + (size_t)kp1 * K;
        stage_vecs([&](int jj) { return h3 + ((size_t)t * kp1 + jj) * ldh; }, kp1, K, hs, gsum);
        if (warp <= k) {
            float v = st.finish(hs + (size_t)warp * K, gsum + (size_t)warp * (K / kGS));
#pragma unroll
            for (int o = 1; o < LPR; o <<= 1) v = __fadd_rn(v, __shfl_down_sync(QE_FULL, v, o));   /* parts in order */
            if (lane % LPR == 0) ys[warp][lane / LPR] = v;
        }
        __syncthreads();
        if (warp == 0 && lane < 32 / LPR && r0 + lane < H) {
            float o = 0.0f;
            for (int jj = 0; jj < k; jj++) o = __fadd_rn(o, __fmul_rn(score[t * k + jj], ys[jj][lane]));
            o = __fadd_rn(o, __fmul_rn(qe_sigmoid(logits[(size_t)t * ld_logits + a.E]), ys[k][lane]));
            out[(size_t)t * H + r0 + lane] = o;
        }
    }
};

template <int BITS>
__global__ void __launch_bounds__(17 * 32) decode_down_combine_kernel(QeExpertArgs a, const float *__restrict__ h3,
                                                                      int ldh, const int32_t *__restrict__ idx,
                                                                      const float *__restrict__ score,
                                                                      const float *__restrict__ logits, int ld_logits,
                                                                      int E, int k, float *__restrict__ out) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float ys[17][32];
    (void)E;
    DownUnit<BITS, kDownLanesPerRow> du;
    du.begin(a, idx, k, blockIdx.x, blockIdx.y * kDownRows);   /* codes in flight while the activations are staged */
    du.end(a, h3, ldh, k, score, logits, ld_logits, out, smem, ys);
}

/* ------------------------------------------------------------------ coalesced decode GEMVs
 * The expert stage of a decode step (a few tokens, one (token, slot) pair per unit) with every warp load
 * coalesced: LPR lanes stream a row, each 16 bytes (CPL = 128 / BITS codes, inside one group of 64), so a warp
 * load covers 32 * 16 contiguous bytes: RPW = 32 / LPR rows when a row is shorter than 512 bytes, or one
 * 512-byte slice of a longer row (NS slices per row, one warp each). A lane's inputs are the same for every row
 * it visits, so its CPL activations and their sum stay in registers; the unit's J row loads are all issued
 * before the first is used. Per load, v = s * 2^b * (sum_i (1 + q_i/2^b) x_i - sum_i x_i) + bias * sum_i x_i
 * over the lane's codes (qmat.c:43 per part of a group: the scale and bias of the group, the dot of its part),
 * then the parts are summed across the row's lanes by a fixed transposed tree and across slices in order. */
constexpr int kDgMaxSlices = 8;
constexpr int kDgGuMaxWarps = 12;   /* gate/up CTA: 2 matrices x slices */
constexpr int kDgDnMaxWarps = 18;   /* down CTA: (k + 1) slots x slices */

/* Lane geometry of a row of K codes: lanes per row (1..32) and slices (rows of at least 512 bytes). */
__host__ __device__ __forceinline__ int dg_lpr(int K, int bits) {
    const int lanes = K * bits / 8 / 16;
    return lanes < 32 ? lanes : 32;
}
__host__ __device__ __forceinline__ int dg_slices(int K, int bits) { return K * bits / 8 / 512; }
/* Supported: every row a power-of-two number (2..16) of 16-byte lanes, or a whole number of 512-byte slices. */
__host__ inline bool dg_supported(int K, int bits) {
    if (K % kGS) return false;
    const int lanes = K * bits / 8 / 16;
    if (lanes >= 32) return lanes % 32 == 0 && lanes / 32 <= kDgMaxSlices;
    return lanes >= 2 && (lanes & (lanes - 1)) == 0;
}

/* One warp's unit: rows r0 + lane / LPR + RPW * j (j < J; rows past `rows` are clamped for the loads and not
 * written) of matrix m for expert e, slice sl, against xv (the K activations in global memory). Returns this
 * lane's reduced value; *row_out is its row, or -1 when the lane does not write. */
template <int BITS, int LPR, int J>
__device__ __forceinline__ float dg_unit(const QeQDev &m, int e, int r0, int sl, const float *__restrict__ xv,
                                         int *row_out) {
    constexpr int CPL = 128 / BITS, RPW = 32 / LPR;
    const int lane = threadIdx.x & 31, rows = m.rows;
    const int kl = (lane % LPR) * CPL + sl * 32 * CPL;          /* first input of this lane */
    const int g = kl / kGS;
    const size_t bpr = (size_t)m.cols * BITS / 8;
    const uint8_t *base = reinterpret_cast<const uint8_t *>(m.w) + (size_t)e * rows * bpr + (size_t)kl * BITS / 8;
    const int ng = m.cols / kGS;
    const size_t so = m.scale_t ? ((size_t)e * ng + g) * rows : (size_t)e * rows * ng + g;
    const size_t sstr = m.scale_t ? 1 : (size_t)ng;             /* between consecutive rows */
    /* codes, scales and biases of the J rows: every load issued before the first use */
    uint4 w[J];
    uint32_t sb[J];
#pragma unroll
    for (int j = 0; j < J; j++) {
        const int row = min(r0 + lane / LPR + RPW * j, rows - 1);
        w[j] = __ldg(reinterpret_cast<const uint4 *>(base + (size_t)row * bpr));
        sb[j] = (uint32_t)__ldg(m.scales + so + row * sstr) | ((uint32_t)__ldg(m.biases + so + row * sstr) << 16);
    }
    /* the lane's activations and their sum (a fixed left-to-right order) */
    float xr[CPL];
    const float4 *x4 = reinterpret_cast<const float4 *>(xv + kl);
#pragma unroll
    for (int i = 0; i < CPL / 4; i++) {
        const float4 t = __ldg(x4 + i);
        xr[4 * i] = t.x; xr[4 * i + 1] = t.y; xr[4 * i + 2] = t.z; xr[4 * i + 3] = t.w;
    }
    float xs = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; i++) xs = __fadd_rn(xs, xr[i]);
    float v[J];
#pragma unroll
    for (int j = 0; j < J; j++) {
        const uint32_t ws[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
        float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            if constexpr (BITS == 4) {
                const float *xq = xr + 8 * q;
                a0 = __ffma2_rn(make_float2(code_v<4, 0>(ws[q]), code_v<4, 1>(ws[q])), make_float2(xq[0], xq[1]), a0);
                a1 = __ffma2_rn(make_float2(code_v<4, 2>(ws[q]), code_v<4, 3>(ws[q])), make_float2(xq[2], xq[3]), a1);
                a0 = __ffma2_rn(make_float2(code_v<4, 4>(ws[q]), code_v<4, 5>(ws[q])), make_float2(xq[4], xq[5]), a0);
                a1 = __ffma2_rn(make_float2(code_v<4, 6>(ws[q]), code_v<4, 7>(ws[q])), make_float2(xq[6], xq[7]), a1);
            } else {
                const float *xq = xr + 4 * q;
                a0 = __ffma2_rn(make_float2(code_v<8, 0>(ws[q]), code_v<8, 1>(ws[q])), make_float2(xq[0], xq[1]), a0);
                a1 = __ffma2_rn(make_float2(code_v<8, 2>(ws[q]), code_v<8, 3>(ws[q])), make_float2(xq[2], xq[3]), a1);
            }
        }
        const float p = __fadd_rn(__fadd_rn(a0.x, a0.y), __fadd_rn(a1.x, a1.y));
        const float sq = __fmul_rn(__fsub_rn(p, xs), (float)(1 << BITS));
        const float s = __uint_as_float(sb[j] << 16), b = __uint_as_float(sb[j] & 0xFFFF0000u);
        v[j] = __fmaf_rn(s, sq, __fmul_rn(b, xs));
    }
    const float r = dg_reduce<LPR, J>(v, lane);
    const int row = r0 + lane / LPR + RPW * dg_index<LPR, J>(lane);
    *row_out = (dg_writer<LPR, J>(lane) && row < rows) ? row : -1;
    return r;
}

/* Rows per unit: J loads of RPW rows. */
template <int LPR, int J>
constexpr int dg_rows() { return J * (32 / LPR); }

/* Gate/up + SwiGLU: CTA = (token-slot pair, block of dg_rows rows); warp (m, sl) = matrix m (gate, up), slice
 * sl; the slices are summed in order, then h = silu(g) * u (ops.c:16-21) -> h3[p][row]. */
template <int BITS, int LPR, int J>
__global__ void __launch_bounds__(kDgGuMaxWarps * 32) dg_gateup_kernel(QeExpertArgs a, const float *__restrict__ x,
                                                                        const int32_t *__restrict__ idx, int k,
                                                                        float *__restrict__ h3, int ldh) {
    constexpr int RU = dg_rows<LPR, J>();
    __shared__ float part[2][kDgMaxSlices][RU];
    const int p = blockIdx.x, t = p / (k + 1), j = p % (k + 1);
    const bool shared = j == k;
    const QeQDev &G = shared ? a.sh_gate : a.gate, &U = shared ? a.sh_up : a.up;
    const int r0 = blockIdx.y * RU;
    if (r0 >= G.rows) return;
    const int e = shared ? 0 : idx[t * k + j];
    const int ns = max(1, dg_slices(a.hidden, BITS)), warp = threadIdx.x >> 5;
    const int m = warp / ns, sl = warp % ns;
    int row;
    const float v = dg_unit<BITS, LPR, J>(m ? U : G, e, r0, sl, x + (size_t)t * a.hidden, &row);
    if (row >= 0) part[m][sl][row - r0] = v;
    __syncthreads();
    if (threadIdx.x < RU && r0 + threadIdx.x < G.rows) {
        float gv = part[0][0][threadIdx.x], uv = part[1][0][threadIdx.x];
        for (int i = 1; i < ns; i++) {
            gv = __fadd_rn(gv, part[0][i][threadIdx.x]);
            uv = __fadd_rn(uv, part[1][i][threadIdx.x]);
        }
        h3[(size_t)p * ldh + r0 + threadIdx.x] = qe_silu_mul(gv, uv);
    }
}

/* Down + combine: CTA = (token, block of dg_rows output rows); warp (slot, sl) = slot (k routed experts, then the
 * shared one), slice sl; slices summed in order, then out = sum_j score_j y_j (slot order) + sigmoid(shared-gate
 * logit) y_shared (moe_layer.c:79-88). */
template <int BITS, int LPR, int J>
__global__ void __launch_bounds__(kDgDnMaxWarps * 32) dg_down_kernel(QeExpertArgs a, const float *__restrict__ h3, int ldh,
                                                        const int32_t *__restrict__ idx,
                                                        const float *__restrict__ score,
                                                        const float *__restrict__ logits, int ld_logits, int k,
                                                        float *__restrict__ out) {
    constexpr int RU = dg_rows<LPR, J>();
    extern __shared__ float ys[];                   /* [k + 1][ns][RU] */
    const int t = blockIdx.x, H = a.hidden, r0 = blockIdx.y * RU, kp1 = k + 1;
    const int ns = max(1, dg_slices(a.inter, BITS)), warp = threadIdx.x >> 5;
    const int j = warp / ns, sl = warp % ns;
    if (j < kp1) {
        const bool shared = j == k;
        int row;
        const float v = dg_unit<BITS, LPR, J>(shared ? a.sh_down : a.down, shared ? 0 : idx[t * k + j], r0, sl,
                                              h3 + ((size_t)t * kp1 + j) * ldh, &row);
        if (row >= 0) ys[((size_t)j * ns + sl) * RU + row - r0] = v;
    }
    __syncthreads();
    const int i = threadIdx.x;
    if (i < RU && r0 + i < H) {
        float o = 0.0f, ysh = 0.0f;
        for (int jj = 0; jj < kp1; jj++) {
            float y = ys[((size_t)jj * ns) * RU + i];
            for (int s2 = 1; s2 < ns; s2++) y = __fadd_rn(y, ys[((size_t)jj * ns + s2) * RU + i]);
            if (jj < k) o = __fadd_rn(o, __fmul_rn(score[t * k + jj], y));
            else ysh = y;
        }
        o = __fadd_rn(o, __fmul_rn(qe_sigmoid(logits[(size_t)t * ld_logits + a.E]), ysh));
        out[(size_t)t * H + r0 + i] = o;
    }
}

/* y = W x for one activation vector and a plain quantized matrix (the whole-model trunk's projections and LM
 * head): CTA = a block of dg_rows rows, one warp per 512-byte slice of the rows; slices summed in order. */
constexpr int kDgMvMaxWarps = 8;
template <int BITS, int LPR, int J>
__global__ void __launch_bounds__(kDgMvMaxWarps * 32) dg_matvec_kernel(QeQDev m, const float *__restrict__ x,
                                                                      float *__restrict__ y) {
    constexpr int RU = dg_rows<LPR, J>();
    __shared__ float part[kDgMvMaxWarps][RU];
    const int r0 = blockIdx.x * RU;
    const int ns = max(1, dg_slices(m.cols, BITS)), sl = threadIdx.x >> 5;
    int row;
    const float v = dg_unit<BITS, LPR, J>(m, 0, r0, sl, x, &row);
    if (row >= 0) part[sl][row - r0] = v;
    __syncthreads();
    const int i = threadIdx.x;
    if (i < RU && r0 + i < m.rows) {
        float acc = part[0][i];
        for (int q = 1; q < ns; q++) acc = __fadd_rn(acc, part[q][i]);
        y[r0 + i] = acc;
    }
}

/* ------------------------------------------------------------------ fused decode step */

__device__ int g_decode_error;   /* first grid-barrier timeout code, read by qe_decode_error() */

/* Grid-wide barrier of a cooperative launch (every CTA resident): arrive on bar[0], the last arrival resets it
 * and advances the generation bar[1]; waiters poll the generation for at most QE_WAIT_NS. Returns false (and
 * records `code`) on timeout. Every thread of the CTA calls it. */
__device__ bool grid_sync(unsigned *bar, int code, int *ok_s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned *gen = bar + 1;
        const unsigned g = *gen;
        __threadfence();
        int ok = 1;
        if (atomicAdd(bar, 1u) + 1u == gridDim.x) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const uint64_t t0 = decode_timer_ns();
            while (*gen == g) {
                if (decode_timer_ns() - t0 > QE_DECODE_WAIT_NS) {
                    ok = 0;
                    atomicCAS(&g_decode_error, 0, code);
                    break;
                }
            }
        }
        __threadfence();
        *ok_s = ok;
    }
    __syncthreads();
    return *ok_s != 0;
}

struct FusedArgs {
    QeExpertArgs a;
    const float *W, *bias;      /* fp32 router [E+1][hidden] (row E: shared-expert gate), bias [E] or null */
    const float *x;             /* [T][hidden] */
    int T, vec;
    float *logits;              /* [T][E+1] */
    int32_t *idx;               /* [T][k] (written by CTA 0) */
    float *score;               /* [T][k] (written by CTA 0) */
    float *h3;                  /* [T*(k+1)][ldh] */
    int ldh;
    float *out;                 /* [T][hidden] */
    unsigned *bar;              /* [2] grid barrier, zero at launch */
};

/* One decode step in one cooperative launch (one CTA of 512 threads per SM):
 *   1. router logits: one warp per router row (route_dev.cuh), rows spread over every warp of the grid;
 *   2. grid barrier; every CTA computes the softmax/top-k of each token itself (warp t: token t; identical
 *      code and inputs, so identical results) into shared memory, CTA 0 also to idx/score;
 *   3. gate/up + SwiGLU units (token-slot pair, 32 rows) spread over the CTAs; each CTA then requests the codes
 *      of its first down unit (the slots' experts are known from step 2);
 *   4. grid barrier (h3 complete); down + combine units (token, 32 output rows).
 * Each phase's work is the standalone kernels' (router_gemv_f32_kernel, route_topk_kernel, decode_gateup_kernel,
 * decode_down_combine_kernel), so the results are bit-identical to the four-launch path. */
template <int BITS>
__global__ void __launch_bounds__(kGuThreads, 1) decode_fused_kernel(const __grid_constant__ FusedArgs f) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float part_sum[2 * kParts][32];
    __shared__ int32_t s_idx[kFusedMaxTokens * 16];
    __shared__ float s_score[kFusedMaxTokens * 16];
    __shared__ int ok_s;
    const QeExpertArgs &a = f.a;
    const int E = a.E, k = a.k, kp1 = k + 1, T = f.T, H = a.hidden, I = a.inter;
    const int warp = threadIdx.x >> 5;
    constexpr int kWarps = kGuThreads / 32;
    /* 1. router: row r on warp r / gridDim.x of CTA r % gridDim.x (every SM streams its share) */
    for (int row = warp * gridDim.x + blockIdx.x; row <= E; row += gridDim.x * kWarps)
        router_row_f32(f.W, f.bias, f.x, T, H, E, row, f.logits, f.vec);
    if (!grid_sync(f.bar, 1, &ok_s)) return;
    /* 2. top-k, per CTA */
    if (warp < T) {
        float *probs_s = smem + (size_t)warp * 2 * E;
        int *idx_s = reinterpret_cast<int *>(probs_s + E);
        route_topk_warp(f.logits + (size_t)warp * (E + 1), warp, E, k, probs_s, idx_s,
                        blockIdx.x == 0 ? f.idx : s_idx, blockIdx.x == 0 ? f.score : s_score, nullptr);
    }
    __syncthreads();
    if (blockIdx.x == 0) {   /* CTA 0 wrote to global memory: copy to its shared arrays */
        for (int i = threadIdx.x; i < T * k; i += blockDim.x) {
            s_idx[i] = f.idx[i];
            s_score[i] = f.score[i];
        }
        __syncthreads();
    }
    /* 3. gate/up + SwiGLU */
    const int nrb = I / 32, units3 = T * kp1 * nrb;
    for (int u = blockIdx.x; u < units3; u += gridDim.x) {
        gateup_unit<BITS>(a, f.x, s_idx, k, f.h3, f.ldh, u / nrb, (u % nrb) * 32, smem, part_sum);
        __syncthreads();   /* shared memory is restaged by the next unit */
    }
    /* 4. down + combine; the first unit's codes are requested before the barrier */
    const int nrd = H / kDownRows, units4 = T * nrd;   /* the same units as decode_down_combine_kernel's CTAs */
    float (*ys)[32] = part_sum;
    DownUnit<BITS, kDownLanesPerRow> du;
    int u = blockIdx.x;
    if (u < units4) du.begin(a, s_idx, k, u / nrd, (u % nrd) * kDownRows);
    if (!grid_sync(f.bar, 2, &ok_s)) return;
    for (; u < units4; u += gridDim.x) {
        if (u != (int)blockIdx.x) du.begin(a, s_idx, k, u / nrd, (u % nrd) * kDownRows);
        du.end(a, f.h3, f.ldh, k, s_score, f.logits, E + 1, f.out, smem, ys);
        __syncthreads();
    }
}

}  // namespace

/* Whether the decode GEMVs cover this block: group size 64, 4- or 8-bit, rows of whole 128-byte chunks (the
 * gate/up rows in at least kParts of them), top_k <= 16, and the shared expert as wide as a routed one. */
bool qe_decode_supported(const QeExpertArgs *a) {
    const int bits = a->gate.bits;
    if (a->gate.group_size != kGS || (bits != 4 && bits != 8)) return false;
    if (a->inter != a->sh_inter || a->k > 16) return false;
    const int bh = a->hidden * bits / 8, bi = a->inter * bits / 8;
    return bh % kChunk == 0 && bh / kChunk >= kParts && bi % kChunk == 0 && a->inter % 4 == 0;
}

template <int BITS, int LPR, int J>
struct DgMatvecLaunch {
    static void run(const QeQDev *m, const float *x, float *y, int ns, cudaStream_t s) {
        constexpr int RU = dg_rows<LPR, J>();
        dg_matvec_kernel<BITS, LPR, J><<<(m->rows + RU - 1) / RU, ns * 32, 0, s>>>(*m, x, y);
    }
};

/* The coalesced GEMVs' launch, dispatched on the lanes per row (a template parameter). */
template <int BITS, template <int, int, int> class Launch, int JMAX, typename... Args>
static void dg_dispatch(int lpr, Args... args) {
    switch (lpr) {
    case 32: Launch<BITS, 32, JMAX>::run(args...); break;
    case 16: Launch<BITS, 16, (JMAX < 16 ? JMAX : 16)>::run(args...); break;
    case 8: Launch<BITS, 8, 8>::run(args...); break;
    case 4: Launch<BITS, 4, 4>::run(args...); break;
    default: Launch<BITS, 2, 2>::run(args...); break;
    }
}
/* loads per lane and unit: for gate/up (12 warps at most, 170 registers) 8 with 4-bit codes (twice the warps of 16:
 * C1 steps 31.2 -> 29.9 us) and 16 with 8-bit codes (C3 decode 59.2 us against 67.6 with 8), measured on one
 * B200; 8 for the down projection (18 warps, 113 registers) */
constexpr int kDgGuLoads4 = 8, kDgGuLoads8 = 16, kDgDnLoads = 8;
template <int BITS, int LPR, int J>
struct DgGateupLaunch {
    static void run(const QeExpertArgs *a, const float *x, const int32_t *idx, int T, float *h3, int ldh, int ns,
                    cudaStream_t s) {
        constexpr int RU = dg_rows<LPR, J>();
        const dim3 grid(T * (a->k + 1), (std::max(a->inter, a->sh_inter) + RU - 1) / RU);
        dg_gateup_kernel<BITS, LPR, J><<<grid, 2 * ns * 32, 0, s>>>(*a, x, idx, a->k, h3, ldh);
    }
};
template <int BITS, int LPR, int J>
struct DgDownLaunch {
    static void run(const QeExpertArgs *a, const float *h3, int ldh, const int32_t *idx, const float *score,
                    const float *logits, int ld_logits, int T, float *out, int ns, cudaStream_t s) {
        constexpr int RU = dg_rows<LPR, J>();
        const int kp1 = a->k + 1;
        const dim3 grid(T, (a->hidden + RU - 1) / RU);
        dg_down_kernel<BITS, LPR, J><<<grid, kp1 * ns * 32, sizeof(float) * kp1 * ns * RU, s>>>(
            *a, h3, ldh, idx, score, logits, ld_logits, a->k, out);
    }
};
static bool dg_off() {
    static const bool off = getenv("QE_DECODE_V1") && strcmp(getenv("QE_DECODE_V1"), "0") != 0;
    return off;
}

/* y = W x (one vector) on the coalesced GEMV: 1 when the shape is not covered (the caller then uses
 * qe_launch_qmatvec), 0 launched, -1 error. */
int qe_launch_dg_matvec(const QeQDev *m, const float *x, float *y, cudaStream_t s) {
    const int bits = m->bits, K = m->cols;
    if (dg_off() || (bits != 4 && bits != 8) || m->group_size != kGS || !dg_supported(K, bits)) return 1;
    const int ns = std::max(1, dg_slices(K, bits));
    if (ns > kDgMvMaxWarps) return 1;
    if (bits == 4) dg_dispatch<4, DgMatvecLaunch, kDgGuLoads4>(dg_lpr(K, 4), m, x, y, ns, s);
    else dg_dispatch<8, DgMatvecLaunch, kDgGuLoads8>(dg_lpr(K, 8), m, x, y, ns, s);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_decode_gateup(const QeExpertArgs *a, const float *x, const int32_t *idx, int T, float *h3, int ldh,
                            cudaStream_t s) {
    const int bits = a->gate.bits, K = a->hidden;
    if (!dg_off() && (bits == 4 || bits == 8) && a->gate.group_size == kGS && dg_supported(K, bits) &&
        2 * std::max(1, dg_slices(K, bits)) <= kDgGuMaxWarps) {
        const int ns = std::max(1, dg_slices(K, bits));
        if (bits == 4) dg_dispatch<4, DgGateupLaunch, kDgGuLoads4>(dg_lpr(K, 4), a, x, idx, T, h3, ldh, ns, s);
        else dg_dispatch<8, DgGateupLaunch, kDgGuLoads8>(dg_lpr(K, 8), a, x, idx, T, h3, ldh, ns, s);
        QE_CHECK(cudaGetLastError());
        return 0;
    }
    if (!qe_decode_supported(a)) QE_FAIL("decode gate/up: unsupported shape");
    dim3 grid(T * (a->k + 1), (a->inter + 31) / 32);
    const size_t smem = sizeof(float) * ((size_t)a->hidden + a->hidden / kGS);
    if (a->gate.bits == 4)
        decode_gateup_kernel<4><<<grid, 2 * kParts * 32, smem, s>>>(*a, x, idx, a->k, h3, ldh);
    else
        decode_gateup_kernel<8><<<grid, 2 * kParts * 32, smem, s>>>(*a, x, idx, a->k, h3, ldh);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_decode_down_combine(const QeExpertArgs *a, const float *h3, int ldh, const int32_t *idx,
                                  const float *score, const float *logits, int ld_logits, int T, float *out,
                                  cudaStream_t s) {
    {
        const int bits = a->down.bits, K = a->inter, ns = std::max(1, dg_slices(a->inter, a->down.bits));
        if (!dg_off() && (bits == 4 || bits == 8) && a->down.group_size == kGS && a->sh_inter == K &&
            dg_supported(K, bits) && (a->k + 1) * ns <= kDgDnMaxWarps) {
            if (bits == 4)
                dg_dispatch<4, DgDownLaunch, kDgDnLoads>(dg_lpr(K, 4), a, h3, ldh, idx, score, logits, ld_logits, T, out, ns, s);
            else
                dg_dispatch<8, DgDownLaunch, kDgDnLoads>(dg_lpr(K, 8), a, h3, ldh, idx, score, logits, ld_logits, T, out, ns, s);
            QE_CHECK(cudaGetLastError());
            return 0;
        }
    }
    if (!qe_decode_supported(a)) QE_FAIL("decode down: unsupported shape");
    const int K = a->inter, kp1 = a->k + 1;
    dim3 grid(T, (a->hidden + kDownRows - 1) / kDownRows);
    const size_t smem = sizeof(float) * (size_t)kp1 * ((size_t)K + K / kGS);
    if (smem > 200 * 1024) QE_FAIL("decode down: %zu B of shared memory", smem);
    if (a->gate.bits == 4) {
        QE_CHECK(qe_set_smem((const void *)decode_down_combine_kernel<4>, smem));
        decode_down_combine_kernel<4><<<grid, kp1 * 32, smem, s>>>(*a, h3, ldh, idx, score, logits, ld_logits, a->E,
                                                                   a->k, out);
    } else {
        QE_CHECK(qe_set_smem((const void *)decode_down_combine_kernel<8>, smem));
        decode_down_combine_kernel<8><<<grid, kp1 * 32, smem, s>>>(*a, h3, ldh, idx, score, logits, ld_logits, a->E,
                                                                   a->k, out);
    }
    QE_CHECK(cudaGetLastError());
    return 0;
}

/* The fused decode step (decode_fused_kernel): fp32 router, T <= kFusedMaxTokens tokens, at most 15 routed
 * slots. Returns 1 (nothing launched) when the shape or the device does not allow it, 0 when launched, -1 on
 * error. bar: two unsigned words of device memory, zeroed here before the launch. */
int qe_launch_decode_fused(const QeExpertArgs *a, const float *W, const float *bias, const float *x, int T,
                           float *logits, int32_t *idx, float *score, float *h3, int ldh, float *out, unsigned *bar,
                           int sms, cudaStream_t s) {
    const int E = a->E, k = a->k, H = a->hidden, I = a->inter;
    if (!qe_decode_supported(a) || T < 1 || T > kFusedMaxTokens || k + 1 > 2 * kParts || E > 32 * kMaxEPL ||
        H > 32 * kRouterLaneChunks * kRouterChunk || H % 32 || I % 32 || k > E)
        return 1;
    const int vec = H % 4 == 0 && ((uintptr_t)W | (uintptr_t)x) % 16 == 0;
    size_t smem = sizeof(float) * (size_t)T * 2 * E;
    smem = std::max(smem, sizeof(float) * ((size_t)H + H / kGS));
    smem = std::max(smem, sizeof(float) * (size_t)(k + 1) * ((size_t)I + I / kGS));
    if (smem > 200 * 1024) return 1;
    const void *kern = a->gate.bits == 4 ? (const void *)decode_fused_kernel<4> : (const void *)decode_fused_kernel<8>;
    QE_CHECK(qe_set_smem(kern, smem));
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGuThreads, smem) != cudaSuccess || per_sm < 1)
        return 1;
    FusedArgs f;
    f.a = *a; f.W = W; f.bias = bias; f.x = x; f.T = T; f.vec = vec; f.logits = logits; f.idx = idx;
    f.score = score; f.h3 = h3; f.ldh = ldh; f.out = out; f.bar = bar;
    QE_CHECK(cudaMemsetAsync(bar, 0, 2 * sizeof(unsigned), s));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);   /* one CTA per SM, all resident (cooperative) */
    cfg.blockDim = dim3(kGuThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a->gate.bits == 4) QE_CHECK(cudaLaunchKernelEx(&cfg, decode_fused_kernel<4>, f));
    else QE_CHECK(cudaLaunchKernelEx(&cfg, decode_fused_kernel<8>, f));
    return 0;
}

int qe_decode_error(void) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_decode_error, sizeof(int)) != cudaSuccess) return -1;
    return v;
}

int qe_decode_error_reset(void) {
    const int zero = 0;
    return cudaMemcpyToSymbol(g_decode_error, &zero, sizeof(int)) == cudaSuccess ? 0 : -1;
}
