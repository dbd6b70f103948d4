/* group_gemv.cu: the expert stage of a batched decode step (a few tokens per expert) as expert-centric
 * CUDA-core GEMVs.
 *
 * Reference: engine/src/moe_layer.c:20-26 (mlp: gate, up, silu*up, down), engine/src/qmat.c:15-49 (per row,
 * per group of 64: scale*sum(q*x) + bias*sum(x)), engine/src/qgroup.c (code j of a group at bit
 * (j % (32/bits))*bits of word j / (32/bits), LSB first). The reference runs one token at a time; here the
 * tokens of a batch are bucketed by expert (bucket.cu) and every active expert's rows are streamed from HBM
 * once per chunk of up to kNT of its tokens, each code converted once and dotted with all of them.
 *
 *   group_gateup_kernel  CTA = (expert, chunk of <= kNT tokens, 32 rows); warps 0-3 stream the gate rows,
 *                        4-7 the up rows, each warp a quarter of K, one lane per row; parts summed in order,
 *                        h = silu(g) * u per (token, row) -> h3[pair][row]
 *   group_down_kernel    CTA = (expert, chunk, 32 output rows); 4 warps split K; y -> ybuf[pair][row], summed
 *                        per token by the combine kernel in slot order
 * A lane streams its row in 64-byte chunks (4 x 16-byte loads; the warp's 32 rows are 32 such streams) through
 * a 2-deep register ring with the chunk's scales and biases; the first loads are issued before the tokens'
 * vectors are staged in shared memory (reads there are broadcasts). Codes are formed as 1 + q/2^b floats and
 * the group sum of x subtracted, as in decode.cu; fp32 throughout (tolerance 1e-5 rel-L2).
 */
#include "qe_common.cuh"
#include "qe_kernels.h"

namespace {

constexpr int kGS = 64;
constexpr int kNT = 4;                 /* tokens per chunk */
constexpr int kChunk = 64;             /* bytes a lane loads per ring slot */
constexpr int kU4 = kChunk / 16;
constexpr int kGuParts = 4;            /* K parts per matrix, gate/up kernel */
constexpr int kDnParts = 4;            /* K parts, down kernel */

/* Code I of word w as the float 1 + q/2^b: the code's bits become the top mantissa bits. */
template <int BITS, int I>
__device__ __forceinline__ float code_v(uint32_t w) {
    constexpr int kTop = 23 - BITS;
    constexpr int kSh = kTop - BITS * I;
    constexpr uint32_t kMask = ((1u << BITS) - 1u) << kTop;
    const uint32_t s = kSh >= 0 ? (w << (kSh >= 0 ? kSh : 0)) : (w >> (kSh < 0 ? -kSh : 0));
    return __uint_as_float((s & kMask) | 0x3F800000u);
}

/* One lane's row: chunks [c0, c1) of codes with their groups' scales and biases, a 2-deep register ring. */
template <int BITS>
struct Stream {
    static constexpr int GB = 64 * BITS / 8;        /* bytes per group */
    static constexpr int GPC = kChunk / GB;         /* groups per chunk */
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
    /* acc[n] += scale*sum_q + bias*sum_x over the chunk's groups (group order), for the nt vectors
     * xs[n*ldx ..] with group sums gs[n*ldg ..] */
    __device__ __forceinline__ void chunk(int slot, int c, const float *xs, int ldx, const float *gs, int ldg, int nt,
                                          float (&acc)[kNT]) const {
#pragma unroll
        for (int gi = 0; gi < GPC; gi++) {
            const int g = c * GPC + gi;
            float2 a[kNT];
#pragma unroll
            for (int n = 0; n < kNT; n++) a[n] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < GB / 16; i++) {
                const uint4 wv = w[slot][gi * (GB / 16) + i];
                const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
                const int k0 = g * 64 + i * (128 / BITS);   /* first input of this 16-byte word */
#pragma unroll
                for (int qd = 0; qd < 4; qd++) {
                    constexpr int CPW = 32 / BITS;          /* codes per 32-bit word */
                    float2 cv[CPW / 2];
#pragma unroll
                    for (int h = 0; h < CPW / 2; h++) {
                        if constexpr (BITS == 4) {
                            const uint32_t x = ws[qd];
                            cv[h] = make_float2(h == 0 ? code_v<4, 0>(x) : h == 1 ? code_v<4, 2>(x) : h == 2 ? code_v<4, 4>(x) : code_v<4, 6>(x),
                                                h == 0 ? code_v<4, 1>(x) : h == 1 ? code_v<4, 3>(x) : h == 2 ? code_v<4, 5>(x) : code_v<4, 7>(x));
                        } else {
                            const uint32_t x = ws[qd];
                            cv[h] = make_float2(h == 0 ? code_v<8, 0>(x) : code_v<8, 2>(x),
                                                h == 0 ? code_v<8, 1>(x) : code_v<8, 3>(x));
                        }
                    }
#pragma unroll
                    for (int n = 0; n < kNT; n++) {
                        if (n < nt) {
                            const float4 *x4 = reinterpret_cast<const float4 *>(xs + (size_t)n * ldx + k0 + qd * CPW);
#pragma unroll
                            for (int h = 0; h < CPW / 4; h++) {
                                const float4 xv = x4[h];
                                a[n] = __ffma2_rn(cv[2 * h], make_float2(xv.x, xv.y), a[n]);
                                a[n] = __ffma2_rn(cv[2 * h + 1], make_float2(xv.z, xv.w), a[n]);
                            }
                        }
                    }
                }
            }
            const float s = __uint_as_float(sb[slot][gi] << 16), b = __uint_as_float(sb[slot][gi] & 0xFFFF0000u);
#pragma unroll
            for (int n = 0; n < kNT; n++) {
                if (n < nt) {
                    const float gsum = gs[(size_t)n * ldg + g];
                    const float sq = __fmul_rn(__fsub_rn(__fadd_rn(a[n].x, a[n].y), gsum), (float)(1 << BITS));
                    acc[n] = __fadd_rn(acc[n], __fmaf_rn(s, sq, __fmul_rn(b, gsum)));
                }
            }
        }
    }
    __device__ __forceinline__ void finish(const float *xs, int ldx, const float *gs, int ldg, int nt,
                                           float (&acc)[kNT]) {
        for (int c = c0; c < c1; c += 2) {
            chunk(0, c, xs, ldx, gs, ldg, nt, acc);
            if (c + 2 < c1) load(0, c + 2);
            if (c + 1 < c1) {
                chunk(1, c + 1, xs, ldx, gs, ldg, nt, acc);
                if (c + 3 < c1) load(1, c + 3);
            }
        }
    }
};

/* The quantized matrix (routed expert e, or the shared one) as row pointers. */
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

/* n vectors of K floats into shared memory (vs[j*K + c]) and their sums per group of 64 (gs[j*(K/64) + g]):
 * one warp per group, lanes add pairs, then a fixed shuffle tree. */
template <typename Src>
__device__ void stage_vecs(Src src, int n, int K, float *vs, float *gs) {
    for (int i = threadIdx.x; i < n * (K / 4); i += blockDim.x) {
        const int j = i / (K / 4), c = i % (K / 4);
        reinterpret_cast<float4 *>(vs + (size_t)j * K)[c] = reinterpret_cast<const float4 *>(src(j))[c];
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

struct GItem {
    int e, off, n0, nt, r0;
    bool shared;
};

/* Work item -> (expert, token chunk, 32-row tile), from the bucket lists (same decomposition as the
 * tensor-core kernels: items of a slot are tile-major, chunk-minor). */
__device__ __forceinline__ GItem gitem(const QeBuckets &b, const int32_t *prefix, int na, int E, int item) {
    int lo = 0, hi = na;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= item) lo = mid; else hi = mid;
    }
    GItem it;
    it.e = b.slot_expert[lo];
    it.shared = it.e == E;
    const int cnt = b.counts[it.e];
    it.off = b.offsets[it.e];
    const int ntn = (cnt + kNT - 1) / kNT;
    const int local = item - prefix[lo];
    it.r0 = (local / ntn) * 32;
    it.n0 = (local % ntn) * kNT;
    it.nt = min(kNT, cnt - it.n0);
    return it;
}

template <int BITS>
__global__ void __launch_bounds__(2 * kGuParts * 32, 2) group_gateup_kernel(QeExpertArgs a, const float *__restrict__ x,
                                                                            QeBuckets b, int kp1,
                                                                            float *__restrict__ h3, int ldh) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float part[2 * kGuParts][kNT][32];
    const int na = b.n_active[0], nitems = b.n_active[1];
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const GItem it = gitem(b, b.slot_items, na, a.E, item);
    const QeQDev &G = it.shared ? a.sh_gate : a.gate, &U = it.shared ? a.sh_up : a.up;
    const int rows = G.rows, K = G.cols, e = it.shared ? 0 : it.e;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = warp / kGuParts, pt = warp % kGuParts;
    const int row = min(it.r0 + lane, rows - 1);
    const int nch = K * BITS / 8 / kChunk;
    const QRow q = qrow(m ? U : G, e, row);
    Stream<BITS> st;
    st.row = q.codes; st.sc = q.sc; st.bi = q.bi; st.gstride = q.gstride;
    st.c0 = pt * nch / kGuParts;
    st.c1 = (pt + 1) * nch / kGuParts;
    st.start();                               /* codes in flight while the tokens' vectors are staged */
    float *xs = smem, *gs = smem + (size_t)kNT * K;
    stage_vecs([&](int j) { return x + (size_t)(b.pairs[it.off + it.n0 + j] / kp1) * K; }, it.nt, K, xs, gs);
    float acc[kNT];
#pragma unroll
    for (int n = 0; n < kNT; n++) acc[n] = 0.0f;
    st.finish(xs, K, gs, K / kGS, it.nt, acc);
#pragma unroll
    for (int n = 0; n < kNT; n++) part[warp][n][lane] = acc[n];
    __syncthreads();
    /* thread (n, lane): token n of the chunk, row r0 + lane; parts summed in order, then SwiGLU (ops.c:16-21) */
    const int n = threadIdx.x >> 5;
    if (n < it.nt && it.r0 + lane < rows) {
        float g = 0.0f, u = 0.0f;
        for (int i = 0; i < kGuParts; i++) {
            g = __fadd_rn(g, part[i][n][lane]);
            u = __fadd_rn(u, part[kGuParts + i][n][lane]);
        }
        const int pid = b.pairs[it.off + it.n0 + n];
        h3[(size_t)pid * ldh + it.r0 + lane] = qe_silu_mul(g, u);
    }
    __syncthreads();   /* shared memory is restaged by the next item */
    }
}

template <int BITS>
__global__ void __launch_bounds__(kDnParts * 32) group_down_kernel(QeExpertArgs a, const float *__restrict__ h3,
                                                                   int ldh, QeBuckets b, float *__restrict__ ybuf) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float part[kDnParts][kNT][32];
    const int na = b.n_active[0], nitems = b.n_active[2];
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const GItem it = gitem(b, b.slot_items + (a.E + 2), na, a.E, item);
    const QeQDev &D = it.shared ? a.sh_down : a.down;
    const int H = D.rows, K = D.cols, e = it.shared ? 0 : it.e;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = min(it.r0 + lane, H - 1);
    const int nch = K * BITS / 8 / kChunk;
    const QRow q = qrow(D, e, row);
    Stream<BITS> st;
    st.row = q.codes; st.sc = q.sc; st.bi = q.bi; st.gstride = q.gstride;
    st.c0 = warp * nch / kDnParts;
    st.c1 = (warp + 1) * nch / kDnParts;
    st.start();
    float *hs = smem, *gs = smem + (size_t)kNT * K;
    stage_vecs([&](int j) { return h3 + (size_t)b.pairs[it.off + it.n0 + j] * ldh; }, it.nt, K, hs, gs);
    float acc[kNT];
#pragma unroll
    for (int n = 0; n < kNT; n++) acc[n] = 0.0f;
    st.finish(hs, K, gs, K / kGS, it.nt, acc);
#pragma unroll
    for (int n = 0; n < kNT; n++) part[warp][n][lane] = acc[n];
    __syncthreads();
    for (int n = warp; n < it.nt; n += kDnParts) {
        if (it.r0 + lane >= H) continue;
        float y = 0.0f;
        for (int i = 0; i < kDnParts; i++) y = __fadd_rn(y, part[i][n][lane]);
        ybuf[(size_t)b.pairs[it.off + it.n0 + n] * H + it.r0 + lane] = y;
    }
    __syncthreads();   /* shared memory is restaged by the next item */
    }
}

}  // namespace

/* Whether the grouped GEMVs cover this block: group size 64, 4- or 8-bit, every row a whole number of
 * 64-byte chunks (the gate/up rows at least kGuParts of them), 16-byte aligned activation rows. */
bool qe_group_supported(const QeExpertArgs *a) {
    const int bits = a->gate.bits;
    if (a->gate.group_size != kGS || (bits != 4 && bits != 8)) return false;
    const int bh = a->hidden * bits / 8, bi = a->inter * bits / 8, bs = a->sh_inter * bits / 8;
    return bh % kChunk == 0 && bh / kChunk >= kGuParts && bi % kChunk == 0 && bs % kChunk == 0 &&
           a->inter % 4 == 0 && a->sh_inter % 4 == 0;
}

int qe_group_tokens(void) { return kNT; }
int qe_group_rows(void) { return 32; }

/* CTAs of `kern` resident per SM with `smem` bytes of dynamic shared memory (at least 1). */
static int resident(const void *kern, int threads, size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem) != cudaSuccess || n < 1) n = 1;
    return n;
}

/* Gate/up + SwiGLU over the buckets (items: expert x 32-row tile x chunk of kNT tokens) -> h3 [pair][ldh].
 * A persistent grid of `sms` x resident CTAs walks the items (their count is on the device). */
int qe_launch_group_gateup(const QeExpertArgs *a, const float *x, const QeBuckets *b, int sms, float *h3, int ldh,
                           cudaStream_t s) {
    if (!qe_group_supported(a)) QE_FAIL("grouped gate/up: unsupported shape");
    const size_t smem = sizeof(float) * (size_t)kNT * ((size_t)a->hidden + a->hidden / kGS);
    const int threads = 2 * kGuParts * 32;
    if (a->gate.bits == 4) {
        const void *k = (const void *)group_gateup_kernel<4>;
        QE_CHECK(qe_set_smem(k, smem));
        group_gateup_kernel<4><<<sms * resident(k, threads, smem), threads, smem, s>>>(*a, x, *b, a->k + 1, h3, ldh);
    } else {
        const void *k = (const void *)group_gateup_kernel<8>;
        QE_CHECK(qe_set_smem(k, smem));
        group_gateup_kernel<8><<<sms * resident(k, threads, smem), threads, smem, s>>>(*a, x, *b, a->k + 1, h3, ldh);
    }
    QE_CHECK(cudaGetLastError());
    return 0;
}

/* Down projection over the buckets (items: expert x 32-row tile x chunk) -> ybuf [pair][hidden]. */
int qe_launch_group_down(const QeExpertArgs *a, const float *h3, int ldh, const QeBuckets *b, int sms, float *ybuf,
                         cudaStream_t s) {
    if (!qe_group_supported(a)) QE_FAIL("grouped down: unsupported shape");
    const int K = a->inter > a->sh_inter ? a->inter : a->sh_inter;
    const size_t smem = sizeof(float) * (size_t)kNT * ((size_t)K + K / kGS);
    const int threads = kDnParts * 32;
    if (a->gate.bits == 4) {
        const void *k = (const void *)group_down_kernel<4>;
        QE_CHECK(qe_set_smem(k, smem));
        group_down_kernel<4><<<sms * resident(k, threads, smem), threads, smem, s>>>(*a, h3, ldh, *b, ybuf);
    } else {
        const void *k = (const void *)group_down_kernel<8>;
        QE_CHECK(qe_set_smem(k, smem));
        group_down_kernel<8><<<sms * resident(k, threads, smem), threads, smem, s>>>(*a, h3, ldh, *b, ybuf);
    }
    QE_CHECK(cudaGetLastError());
    return 0;
}
