/* expert_mma.cu: quantized expert projections on the tensor cores, for decode and small batches.
 *
 * Reference: engine/src/moe_layer.c:20-26 (mlp: gate, up, silu*up, down), :79-88 (weighted combine and
 * the sigmoid-gated shared expert), engine/src/qmat.c:15-49 (affine dequant, factorised per group as
 * scale*sum(q*x) + bias*sum(x)), engine/src/qgroup.c (code j of a group at bit (j % (32/bits))*bits of
 * word j / (32/bits), LSB first).
 *
 * Precision. The 4- and 8-bit codes are exact in bf16, and the reference's factorisation keeps scale and
 * bias out of the products, so each group's sum(q*x) is computed by bf16 MMAs with fp32 accumulation on
 * x split into three bf16 terms (x = hi + mid + lo, 24 significant bits): the products are exact, and the
 * per-group partial is then scaled in fp32 exactly like qmat.c:41-44. The result agrees with the fp32
 * reference to ~1e-7 relative, far inside the 1e-5 relative-L2 bound.
 *
 * Tiling. One warp owns 16 weight rows x 8 tokens (mma.m16n8k16: A = codes, B = x). Lane (g, t) holds
 * rows g and g+8 and supplies, per k16 step, the logical k positions {2t, 2t+1, 2t+8, 2t+9}. The MMA sums
 * over k in any order, so the columns are permuted so that each lane's codes come from a few contiguous
 * packed words it loads with one 8/16/32-byte vector load per row and group:
 *   4-bit: lane t reads words [(t&1)*S, (t&1)*S + S) of the group (S = GS/16 k16 steps); in step s it
 *          uses word (t&1)*S + s, nibble pairs (n0, n0+4) and (n0+1, n0+5) with n0 = 2*(t>>1);
 *   8-bit: lane t reads words [t*S, t*S + S); in step s it uses word t*S + s, byte pairs (0,2), (1,3).
 * The activations are staged once per CTA in shared memory in exactly that permuted order, already
 * split into the three bf16 terms, so every B fragment is one aligned shared-memory load.
 */
#include "qe_common.cuh"
#include "qe_kernels.h"

namespace {

constexpr int kNT = 8;       /* tokens per MMA (n8) */
constexpr int kWarps = 4;    /* warps per CTA; each warp = 16 rows */
constexpr int kRowsPerCta = 16 * kWarps;
/* Decode-sized batches (T <= kSplitMaxT): the 4 warps of a CTA share 16 rows and split the groups of K
 * between them (partials summed in warp order), so a 1-token step has 4x more CTAs streaming weights. */
constexpr int kSplitMaxT = 4;
constexpr int kSplitK = 4;

enum { MODE_GATEUP = 0, MODE_DOWN = 1 };

template <int BITS, int GS>
struct Geo {
    static constexpr int S = GS / 16;                  /* k16 steps per group, words per lane per row */
    static constexpr int WPG = GS * BITS / 32;         /* packed words per group per row */
    static constexpr int GROUP_U32 = 4 * S * 3 * 2;    /* staged B words per (token, group) */
    __device__ static int lane_word(int t) { return BITS == 4 ? (t & 1) * S : t * S; }
    /* column (within a group) -> lane t, step s, logical position j in {2t, 2t+1, 2t+8, 2t+9} */
    __device__ static void col_pos(int c, int &t, int &s, int &j) {
        if (BITS == 4) {
            const int word = c >> 3, nib = c & 7;
            const int half = word / S;
            s = word % S;
            const int hi2 = (nib >> 1) & 1;     /* nibbles {2,3,6,7} -> t>>1 = 1 */
            t = half | (hi2 << 1);
            const int rel = nib - 2 * hi2;      /* in {0,1,4,5} */
            j = ((rel >> 2) & 1) | ((rel & 1) << 1);
        } else {
            const int word = c >> 2, byte = c & 3;
            t = word / S;
            s = word % S;
            j = ((byte >> 1) & 1) | ((byte & 1) << 1);
        }
    }
};

template <int N>
struct Words { uint32_t v[N]; };

template <int N>
__device__ __forceinline__ Words<N> load_words(const uint32_t *p) {
    Words<N> w;
    if constexpr (N == 2) {
        const uint2 a = __ldg(reinterpret_cast<const uint2 *>(p));
        w.v[0] = a.x; w.v[1] = a.y;
    } else if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N / 4; i++) {
            const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p) + i);
            w.v[4 * i] = a.x; w.v[4 * i + 1] = a.y; w.v[4 * i + 2] = a.z; w.v[4 * i + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; i++) w.v[i] = __ldg(p + i);
    }
    return w;
}

/* bf16x2 pair of codes from one packed word for logical positions (2t, 2t+1) [lo] or (2t+8, 2t+9) [hi] */
template <int BITS>
__device__ __forceinline__ void codes_to_bf16x2(uint32_t w, int t, uint32_t &lo, uint32_t &hi) {
    if constexpr (BITS == 4) {
        const int n0 = (t >> 1) * 2;
        const uint32_t a = ((w >> (4 * n0)) & 0x000F000Fu) | 0x43004300u;
        const uint32_t b = ((w >> (4 * n0 + 4)) & 0x000F000Fu) | 0x43004300u;
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
        __nv_bfloat162 fa = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&a), k128);
        __nv_bfloat162 fb = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&b), k128);
        lo = *reinterpret_cast<uint32_t *>(&fa);
        hi = *reinterpret_cast<uint32_t *>(&fb);
    } else {
        const float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540)) - 8388608.0f;
        const float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541)) - 8388608.0f;
        const float f2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542)) - 8388608.0f;
        const float f3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543)) - 8388608.0f;
        lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f2), 0x7632);
        hi = __byte_perm(__float_as_uint(f1), __float_as_uint(f3), 0x7632);
    }
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

/* Stage nt activation rows (K = cols) into shared memory: split into 3 bf16 terms in the permuted
 * fragment order, plus per-group fp32 sums. Layout per token: [group][lane t][step s][term][2 u32]. */
template <int BITS, int GS>
__device__ void stage_rows(const float *const *rows, int nt, int K, uint32_t *xs, float *xsum, int tstride) {
    using G = Geo<BITS, GS>;
    const int ng = K / GS;
    __nv_bfloat16 *xb = reinterpret_cast<__nv_bfloat16 *>(xs);
    for (int e = threadIdx.x; e < nt * K; e += blockDim.x) {
        const int n = e / K, c = e % K;
        const int g = c / GS, cg = c % GS;
        int t, s, j;
        G::col_pos(cg, t, s, j);
        const float v = rows[n][c];
        __nv_bfloat16 h, m, l;
        qe_split3(v, h, m, l);
        const int base = n * tstride + g * G::GROUP_U32 + ((t * G::S + s) * 3) * 2 + (j >> 1);
        xb[2 * base + (j & 1)] = h;
        xb[2 * (base + 2) + (j & 1)] = m;
        xb[2 * (base + 4) + (j & 1)] = l;
    }
    for (int e = threadIdx.x; e < kNT * ng; e += blockDim.x) {
        const int n = e / ng, g = e % ng;
        float sum = 0.0f;
        if (n < nt)
            for (int i = 0; i < GS; i++) sum = __fadd_rn(sum, rows[n][g * GS + i]);
        xsum[n * ng + g] = sum; /* columns n >= nt are computed but never stored */
    }
}

/* One warp: out[4] (rows g, g+8 x tokens 2t, 2t+1) += W[16 rows] . x over groups [g0, g1), the range's
 * group terms summed from 0 in group order and then added to out. The code words of the next kDepth
 * groups are always in flight (a register ring), so a warp streams its rows instead of waiting one memory
 * latency per group. */
constexpr int kDepth = 4;
template <int BITS, int GS, int NMAT>
__device__ __forceinline__ void warp_qmm(const QeQDev *const mats[NMAT], const size_t row_word[NMAT][2],
                                         const size_t row_grp[NMAT][2], size_t grp_stride, const bool row_ok[2], int g0,
                                         int g1, int ng, const uint32_t *xs, const float *xsum, int tstride, int nt,
                                         float (&acc)[NMAT][4]) {
    using G = Geo<BITS, GS>;
    const int lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
    const int lw = G::lane_word(t);
    const bool tok_ok = gq < nt;
    const uint32_t *xrow = xs + (size_t)gq * tstride + (size_t)t * G::S * 6;
    float pacc[NMAT][4];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++) pacc[m][i] = 0.0f;
    Words<G::S> ring[kDepth][NMAT][2];
    auto fetch = [&](int g, Words<G::S>(&wa)[NMAT][2]) {
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int r = 0; r < 2; r++) {
                if (row_ok[r] && g < g1) {
                    wa[m][r] = load_words<G::S>(mats[m]->w + row_word[m][r] + (size_t)g * G::WPG + lw);
                } else {
#pragma unroll
                    for (int i = 0; i < G::S; i++) wa[m][r].v[i] = 0u;
                }
            }
    };
#pragma unroll
    for (int d = 0; d < kDepth; d++) fetch(g0 + d, ring[d]);
    for (int gb = g0; gb < g1; gb += kDepth)
#pragma unroll
    for (int d = 0; d < kDepth; d++) {
        const int g = gb + d;
        if (g >= g1) break;
        Words<G::S>(&wa)[NMAT][2] = ring[d];
        float p[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int i = 0; i < 4; i++) p[m][i] = 0.0f;
        const uint32_t *xg = xrow + (size_t)g * G::GROUP_U32;
#pragma unroll
        for (int s = 0; s < G::S; s++) {
            uint32_t b[3][2];
#pragma unroll
            for (int term = 0; term < 3; term++) {
                if (tok_ok) {
                    const uint2 bb = *reinterpret_cast<const uint2 *>(xg + (s * 3 + term) * 2);
                    b[term][0] = bb.x;
                    b[term][1] = bb.y;
                } else {
                    b[term][0] = b[term][1] = 0u;
                }
            }
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                uint32_t a0, a1, a2, a3;
                codes_to_bf16x2<BITS>(wa[m][0].v[s], t, a0, a2);  /* row g:   (2t,2t+1), (2t+8,2t+9) */
                codes_to_bf16x2<BITS>(wa[m][1].v[s], t, a1, a3);  /* row g+8 */
#pragma unroll
                for (int term = 0; term < 3; term++) mma_bf16_16816(p[m], a0, a1, a2, a3, b[term][0], b[term][1]);
            }
        }
        /* epilogue of the group: scale*sum_q + bias*sum_x (qmat.c:43) */
        const float xs0 = xsum[(2 * t) * ng + g], xs1 = xsum[(2 * t + 1) * ng + g];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int r = 0; r < 2; r++) {
                float sc = 0.0f, bi = 0.0f;
                if (row_ok[r]) {
                    sc = qe_bf16_to_f32(__ldg(mats[m]->scales + row_grp[m][r] + g * grp_stride));
                    bi = qe_bf16_to_f32(__ldg(mats[m]->biases + row_grp[m][r] + g * grp_stride));
                }
                pacc[m][2 * r] = __fadd_rn(pacc[m][2 * r], __fmaf_rn(sc, p[m][2 * r], __fmul_rn(bi, xs0)));
                pacc[m][2 * r + 1] = __fadd_rn(pacc[m][2 * r + 1], __fmaf_rn(sc, p[m][2 * r + 1], __fmul_rn(bi, xs1)));
            }
        fetch(g + kDepth, ring[d]);
    }
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[m][i] = __fadd_rn(acc[m][i], pacc[m][i]);
}

__device__ __forceinline__ int find_slot(const int32_t *prefix, int n, int item) {
    int lo = 0, hi = n; /* prefix[lo] <= item < prefix[hi] */
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= item) lo = mid; else hi = mid;
    }
    return lo;
}

/* MODE_GATEUP: h3[pair][row] = silu(gate.x) * (up.x)   (moe_layer.c:20-25, ops.c:16-21)
 * MODE_DOWN:   y[pair][row]  = down.h3                  (moe_layer.c:25) */
template <int BITS, int GS, int MODE, int KS>
__global__ void __launch_bounds__(kWarps * 32) expert_kernel(QeExpertArgs a, const float *__restrict__ xin, int ldx,
                                                             QeBuckets bk, int T, float *__restrict__ out,
                                                             int ldo, int chunk) {
    constexpr int kRows = 16 * kWarps / KS;   /* rows per CTA */
    __shared__ float red[KS > 1 ? kWarps * 32 * 8 : 1];
    extern __shared__ __align__(16) uint32_t smem[];
    using G = Geo<BITS, GS>;
    const int Kmax = MODE == MODE_GATEUP ? a.hidden : max(a.inter, a.sh_inter);
    const int tstride = (Kmax / GS) * G::GROUP_U32 + 4;
    uint32_t *xs = smem;
    float *xsum = reinterpret_cast<float *>(smem + (size_t)chunk * tstride);
    __shared__ const float *rows[kNT];
    __shared__ int pair_ids[kNT];
    const int na = bk.n_active[0];
    const int nitems = bk.n_active[MODE == MODE_GATEUP ? 1 : 2];
    const int32_t *prefix = bk.slot_items + (MODE == MODE_GATEUP ? 0 : (a.E + 2));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
    const int kp1 = a.k + 1;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int slot = find_slot(prefix, na, item);
        const int e = bk.slot_expert[slot];
        const bool shared = e == a.E;
        const int count = bk.counts[e], off = bk.offsets[e];
        const int rows_total = MODE == MODE_GATEUP ? (shared ? a.sh_inter : a.inter) : a.hidden;
        const int K = MODE == MODE_GATEUP ? a.hidden : (shared ? a.sh_inter : a.inter);
        const int tiles = (rows_total + kRows - 1) / kRows;
        const int local = item - prefix[slot];
        const int ch = local / tiles, tile = local % tiles;
        const int p0 = ch * chunk;
        const int nt = min(chunk, count - p0);
        __syncthreads(); /* previous item finished with the staging buffers */
        if (threadIdx.x < kNT) {
            const int n = threadIdx.x;
            if (n < nt) {
                const int p = bk.pairs[off + p0 + n];
                pair_ids[n] = p;
                rows[n] = MODE == MODE_GATEUP ? xin + (size_t)(p / kp1) * ldx : xin + (size_t)p * ldx;
            } else {
                pair_ids[n] = -1;
                rows[n] = nullptr;
            }
        }
        __syncthreads();
        stage_rows<BITS, GS>(rows, nt, K, xs, xsum, tstride);
        __syncthreads();
        const int sub = warp / KS, part = warp % KS;
        const int r_base = tile * kRows + sub * 16;
        const int ng = K / GS;
        /* the group ranges of the decode split; a warp that owns all of them runs them in order, so a token's
         * sums are the same whichever kernel variant (batch size) computes them */
        const int q0 = KS > 1 ? part : 0, q1 = KS > 1 ? part + 1 : kSplitK;
        /* KS > 1: the warps of a row block add their partials in warp order into the first one */
        auto reduce_parts = [&](float *accv, int n) {
            if constexpr (KS > 1) {
                for (int i = 0; i < n; i++) red[(warp * 32 + lane) * 8 + i] = accv[i];
                __syncthreads();
                if (part == 0)
                    for (int q = 1; q < KS; q++)
                        for (int i = 0; i < n; i++) accv[i] = __fadd_rn(accv[i], red[((warp + q) * 32 + lane) * 8 + i]);
            }
        };
        const bool row_ok[2] = {r_base + gq < rows_total, r_base + gq + 8 < rows_total};
        if (MODE == MODE_GATEUP) {
            const QeQDev *mats[2] = {shared ? &a.sh_gate : &a.gate, shared ? &a.sh_up : &a.up};
            const size_t wpr = (size_t)K * BITS / 32, gpr = (size_t)K / GS;
            const size_t ebase = shared ? 0 : (size_t)e * rows_total;
            size_t rw[2][2], rg[2][2];
            const size_t eg = shared ? 0 : (size_t)e;
#pragma unroll
            for (int m = 0; m < 2; m++)
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const size_t rin = (size_t)(row_ok[r] ? r_base + gq + 8 * r : 0);
                    rw[m][r] = (ebase + rin) * wpr;
                    rg[m][r] = mats[m]->scale_t ? eg * gpr * rows_total + rin : (ebase + rin) * gpr;
                }
            float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
            for (int q = q0; q < q1; q++)
                warp_qmm<BITS, GS, 2>(mats, rw, rg, mats[0]->scale_t ? (size_t)rows_total : 1, row_ok,
                                      q * ng / kSplitK, (q + 1) * ng / kSplitK, ng, xs, xsum, tstride, nt, acc);
            reduce_parts(&acc[0][0], 8);
#pragma unroll
            for (int r = 0; r < 2; r++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int n = 2 * t + c;
                    if (part == 0 && row_ok[r] && n < nt) {
                        const int row = r_base + gq + 8 * r;
                        out[(size_t)pair_ids[n] * ldo + row] = qe_silu_mul(acc[0][2 * r + c], acc[1][2 * r + c]);
                    }
                }
        } else {
            const QeQDev *mats[1] = {shared ? &a.sh_down : &a.down};
            const size_t wpr = (size_t)K * BITS / 32, gpr = (size_t)K / GS;
            const size_t ebase = shared ? 0 : (size_t)e * rows_total;
            size_t rw[1][2], rg[1][2];
            const size_t eg = shared ? 0 : (size_t)e;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const size_t rin = (size_t)(row_ok[r] ? r_base + gq + 8 * r : 0);
                rw[0][r] = (ebase + rin) * wpr;
                rg[0][r] = mats[0]->scale_t ? eg * gpr * rows_total + rin : (ebase + rin) * gpr;
            }
            float acc[1][4] = {{0, 0, 0, 0}};
            for (int q = q0; q < q1; q++)
                warp_qmm<BITS, GS, 1>(mats, rw, rg, mats[0]->scale_t ? (size_t)rows_total : 1, row_ok,
                                      q * ng / kSplitK, (q + 1) * ng / kSplitK, ng, xs, xsum, tstride, nt, acc);
            reduce_parts(&acc[0][0], 4);
#pragma unroll
            for (int r = 0; r < 2; r++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int n = 2 * t + c;
                    if (part == 0 && row_ok[r] && n < nt) {
                        const int row = r_base + gq + 8 * r;
                        out[(size_t)pair_ids[n] * ldo + row] = acc[0][2 * r + c];
                    }
                }
        }
    }
}

template <int BITS, int GS, int MODE>
int launch_expert(const QeExpertArgs *a, const float *xin, int ldx, const QeBuckets *b, int T, float *out, int ldo,
                  int grid, cudaStream_t s) {
    using G = Geo<BITS, GS>;
    const int Kmax = MODE == MODE_GATEUP ? a->hidden : (a->inter > a->sh_inter ? a->inter : a->sh_inter);
    const int tstride = (Kmax / GS) * G::GROUP_U32 + 4;
    const int chunk = T < kNT ? T : kNT;
    const size_t smem = sizeof(uint32_t) * (size_t)chunk * tstride + sizeof(float) * (size_t)kNT * (Kmax / GS);
    if (smem > 200 * 1024) QE_FAIL("expert kernel: K=%d needs %zu B of shared memory", Kmax, smem);
    auto kern = T <= kSplitMaxT ? expert_kernel<BITS, GS, MODE, kSplitK> : expert_kernel<BITS, GS, MODE, 1>;
    QE_CHECK(qe_set_smem((const void *)kern, smem));
    kern<<<grid, kWarps * 32, smem, s>>>(*a, xin, ldx, *b, T, out, ldo, chunk);
    QE_CHECK(cudaGetLastError());
    return 0;
}

template <int MODE>
int dispatch(const QeExpertArgs *a, const float *xin, int ldx, const QeBuckets *b, int T, float *out, int ldo, int grid,
             cudaStream_t s) {
    const int bits = a->gate.bits, gs = a->gate.group_size;
    if (bits == 4 && gs == 64) return launch_expert<4, 64, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    if (bits == 8 && gs == 64) return launch_expert<8, 64, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    if (bits == 4 && gs == 32) return launch_expert<4, 32, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    if (bits == 4 && gs == 128) return launch_expert<4, 128, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    if (bits == 8 && gs == 32) return launch_expert<8, 32, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    if (bits == 8 && gs == 128) return launch_expert<8, 128, MODE>(a, xin, ldx, b, T, out, ldo, grid, s);
    QE_FAIL("expert kernel: unsupported bits=%d group_size=%d", bits, gs);
}

/* out[t] = sum_i score_i * y_i (top-k order) + sigmoid(gsh) * y_shared   (moe_layer.c:78-88) */
__global__ void combine_kernel(const float *__restrict__ ybuf, const float *__restrict__ score,
                               const float *__restrict__ logits, int ld_logits, int T, int E, int k, int H,
                               float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * H) return;
    const int t = (int)(i / H), j = (int)(i % H);
    const float *y = ybuf + (size_t)t * (k + 1) * H + j;
    float o = 0.0f;
    for (int s = 0; s < k; s++) o = __fadd_rn(o, __fmul_rn(score[(size_t)t * k + s], y[(size_t)s * H]));
    const float sg = qe_sigmoid(logits[(size_t)t * ld_logits + E]);
    o = __fadd_rn(o, __fmul_rn(sg, y[(size_t)k * H]));
    out[i] = o;
}

/* Expert-parallel partial sums (moe_layer.c:79-88 split by owner GPU): out[t] = sum over the routed slots
 * this GPU owns (idx >= 0), in slot order, of score * y, and/or sigmoid(gsh) * y_shared. */
__global__ void combine_sel_kernel(const float *__restrict__ ybuf, const int32_t *__restrict__ idx,
                                   const float *__restrict__ score, const float *__restrict__ logits, int ld_logits,
                                   int T, int E, int k, int H, int with_routed, int with_shared,
                                   float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * H) return;
    const int t = (int)(i / H), j = (int)(i % H);
    const float *y = ybuf + (size_t)t * (k + 1) * H + j;
    float o = 0.0f;
    if (with_routed)
        for (int s = 0; s < k; s++)
            if (idx[(size_t)t * k + s] >= 0) o = __fadd_rn(o, __fmul_rn(score[(size_t)t * k + s], y[(size_t)s * H]));
    if (with_shared) o = __fadd_rn(o, __fmul_rn(qe_sigmoid(logits[(size_t)t * ld_logits + E]), y[(size_t)k * H]));
    out[i] = o;
}

/* y[t][rows] = W x_t for T vectors (qmat_matvec semantics, engine/src/qmat.c:15-49): CTA = 64 rows x
 * 8 vectors, same warp routine as the expert kernels. */
template <int BITS, int GS>
__global__ void __launch_bounds__(kWarps * 32) qmat_kernel(QeQDev m, const float *__restrict__ x, int T,
                                                           float *__restrict__ y) {
    extern __shared__ __align__(16) uint32_t smem[];
    using G = Geo<BITS, GS>;
    const int K = m.cols, ng = K / GS;
    const int tstride = ng * G::GROUP_U32 + 4;
    const int t0 = blockIdx.y * kNT, nt = min(kNT, T - t0);
    const int chunk = min(kNT, T);
    uint32_t *xs = smem;
    float *xsum = reinterpret_cast<float *>(smem + (size_t)chunk * tstride);
    __shared__ const float *rows[kNT];
    if (threadIdx.x < kNT) rows[threadIdx.x] = threadIdx.x < nt ? x + (size_t)(t0 + threadIdx.x) * K : nullptr;
    __syncthreads();
    stage_rows<BITS, GS>(rows, nt, K, xs, xsum, tstride);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
    const int r_base = blockIdx.x * kRowsPerCta + warp * 16;
    const bool row_ok[2] = {r_base + gq < m.rows, r_base + gq + 8 < m.rows};
    const QeQDev *mats[1] = {&m};
    const size_t wpr = (size_t)K * BITS / 32, gpr = (size_t)ng;
    size_t rw[1][2], rg[1][2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const size_t row = (size_t)(row_ok[r] ? r_base + gq + 8 * r : 0);
        rw[0][r] = row * wpr;
        rg[0][r] = m.scale_t ? row : row * gpr;
    }
    float acc[1][4] = {{0, 0, 0, 0}};
    warp_qmm<BITS, GS, 1>(mats, rw, rg, m.scale_t ? (size_t)m.rows : 1, row_ok, 0, ng, ng, xs, xsum, tstride, nt,
                          acc);
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int n = 2 * t + c;
            if (row_ok[r] && n < nt) y[(size_t)(t0 + n) * m.rows + r_base + gq + 8 * r] = acc[0][2 * r + c];
        }
}

template <int BITS, int GS>
int launch_qmat(const QeQDev *m, const float *x, int T, float *y, cudaStream_t s) {
    using G = Geo<BITS, GS>;
    const int ng = m->cols / GS, tstride = ng * G::GROUP_U32 + 4, chunk = T < kNT ? T : kNT;
    const size_t smem = sizeof(uint32_t) * (size_t)chunk * tstride + sizeof(float) * (size_t)kNT * ng;
    if (smem > 200 * 1024) QE_FAIL("qmat: cols=%d needs %zu B of shared memory", m->cols, smem);
    auto kern = qmat_kernel<BITS, GS>;
    QE_CHECK(qe_set_smem((const void *)kern, smem));
    dim3 grid((m->rows + kRowsPerCta - 1) / kRowsPerCta, (T + kNT - 1) / kNT);
    kern<<<grid, kWarps * 32, smem, s>>>(*m, x, T, y);
    QE_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace

int qe_launch_gateup(const QeExpertArgs *a, const float *x, const QeBuckets *b, int T, float *h3, int ldh, int grid,
                     cudaStream_t s) {
    return dispatch<MODE_GATEUP>(a, x, a->hidden, b, T, h3, ldh, grid, s);
}

int qe_launch_down(const QeExpertArgs *a, const float *h3, int ldh, const QeBuckets *b, int T, float *ybuf, int grid,
                   cudaStream_t s) {
    return dispatch<MODE_DOWN>(a, h3, ldh, b, T, ybuf, a->hidden, grid, s);
}

/* Same as combine_kernel, 4 consecutive outputs per thread with 16-byte loads and stores (H % 4 == 0). */
__global__ void combine4_kernel(const float *__restrict__ ybuf, const float *__restrict__ score,
                                const float *__restrict__ logits, int ld_logits, int T, int E, int k, int H,
                                float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;   /* float4 index */
    const int H4 = H / 4;
    if (i >= (long long)T * H4) return;
    const int t = (int)(i / H4), j4 = (int)(i % H4);
    const float4 *y = reinterpret_cast<const float4 *>(ybuf + (size_t)t * (k + 1) * H) + j4;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    /* the slots' rows in batches of 8 independent loads (the shared expert's row with the last batch), then
     * added in slot order */
    const float4 vsh = y[(size_t)k * H4];
    for (int s0 = 0; s0 < k; s0 += 8) {
        float4 v[8];
        float sc[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (s0 + u < k) {
                v[u] = y[(size_t)(s0 + u) * H4];
                sc[u] = score[(size_t)t * k + s0 + u];
            }
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (s0 + u < k) {
                o.x = __fadd_rn(o.x, __fmul_rn(sc[u], v[u].x));
                o.y = __fadd_rn(o.y, __fmul_rn(sc[u], v[u].y));
                o.z = __fadd_rn(o.z, __fmul_rn(sc[u], v[u].z));
                o.w = __fadd_rn(o.w, __fmul_rn(sc[u], v[u].w));
            }
    }
    const float sg = qe_sigmoid(logits[(size_t)t * ld_logits + E]);
    const float4 v = vsh;
    o.x = __fadd_rn(o.x, __fmul_rn(sg, v.x));
    o.y = __fadd_rn(o.y, __fmul_rn(sg, v.y));
    o.z = __fadd_rn(o.z, __fmul_rn(sg, v.z));
    o.w = __fadd_rn(o.w, __fmul_rn(sg, v.w));
    reinterpret_cast<float4 *>(out)[i] = o;
}

int qe_launch_combine(const float *ybuf, const float *score, const float *logits, int ld_logits, int T, int E, int k,
                      int H, float *out, cudaStream_t s) {
    if (H % 4 == 0 && ((uintptr_t)ybuf | (uintptr_t)out) % 16 == 0) {
        const long long n4 = (long long)T * (H / 4);
        combine4_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(ybuf, score, logits, ld_logits, T, E, k, H, out);
        QE_CHECK(cudaGetLastError());
        return 0;
    }
    const long long n = (long long)T * H;
    combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ybuf, score, logits, ld_logits, T, E, k, H, out);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_combine_sel(const float *ybuf, const int32_t *idx, const float *score, const float *logits,
                          int ld_logits, int T, int E, int k, int H, int with_routed, int with_shared, float *out,
                          cudaStream_t s) {
    const long long n = (long long)T * H;
    combine_sel_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ybuf, idx, score, logits, ld_logits, T, E, k, H,
                                                                   with_routed, with_shared, out);
    QE_CHECK(cudaGetLastError());
    return 0;
}

/* Expert parallelism through peer memory: the same partial sums as combine_sel_kernel (routed slots only),
 * each row written straight into its home rank's return buffer. Row t (global row row0 + t of the receive
 * buffer) came from rank s = (row0 + t) / Tblk, slot (row0 + t) % Tblk; it lands at
 * dst_base[s] + (self * Tblk + slot) * H. Rows without a slot of this rank are padding and are skipped. */
__global__ void combine_sel_scatter_kernel(const float *__restrict__ ybuf, const int32_t *__restrict__ idx,
                                           const float *__restrict__ score, int T, int k, int H,
                                           float *const *__restrict__ dst_base, int row0, int Tblk, int self) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * H) return;
    const int t = (int)(i / H), j = (int)(i % H);
    bool any = false;
    for (int s = 0; s < k; s++) any |= idx[(size_t)t * k + s] >= 0;
    if (!any) return;
    const float *y = ybuf + (size_t)t * (k + 1) * H + j;
    float o = 0.0f;
    for (int s = 0; s < k; s++)
        if (idx[(size_t)t * k + s] >= 0) o = __fadd_rn(o, __fmul_rn(score[(size_t)t * k + s], y[(size_t)s * H]));
    const int r = row0 + t, src = r / Tblk, slot = r % Tblk;
    dst_base[src][((size_t)self * Tblk + slot) * H + j] = o;
}

int qe_launch_combine_sel_scatter(const float *ybuf, const int32_t *idx, const float *score, int T, int k, int H,
                                  float *const *dst_base, int row0, int Tblk, int self, cudaStream_t s) {
    const long long n = (long long)T * H;
    combine_sel_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ybuf, idx, score, T, k, H, dst_base, row0,
                                                                           Tblk, self);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_expert_rows_per_cta(int T) { return T <= kSplitMaxT ? kRowsPerCta / kSplitK : kRowsPerCta; }

int qe_launch_qmatvec(const QeQDev *m, const float *x, int T, float *y, cudaStream_t s) {
    const int bits = m->bits, gs = m->group_size;
    if (bits == 4 && gs == 64) return launch_qmat<4, 64>(m, x, T, y, s);
    if (bits == 8 && gs == 64) return launch_qmat<8, 64>(m, x, T, y, s);
    if (bits == 4 && gs == 32) return launch_qmat<4, 32>(m, x, T, y, s);
    if (bits == 4 && gs == 128) return launch_qmat<4, 128>(m, x, T, y, s);
    if (bits == 8 && gs == 32) return launch_qmat<8, 32>(m, x, T, y, s);
    if (bits == 8 && gs == 128) return launch_qmat<8, 128>(m, x, T, y, s);
    QE_FAIL("qmat: unsupported bits=%d group_size=%d", bits, gs);
}
