/* group_gemv.cu: the expert stage of a batched decode step (a few tokens per expert) as expert-centric GEMVs on
 * mma.sync tensor-core fragments.
 *
 * Reference: engine/src/moe_layer.c:20-26 (mlp: gate, up, silu*up, down), engine/src/qmat.c:15-49 (per row,
 * per group of 64: scale*sum(q*x) + bias*sum(x)), engine/src/qgroup.c (code j of a group at bit (j % (32/bits))*bits
 * of word j / (32/bits), LSB first). The reference runs one token at a time; here the tokens of a batch are
 * bucketed by expert (bucket.cu, which also lists each expert's tokens in chunks of up to 4) and every active
 * expert's rows are streamed from HBM once per chunk.
 *
 * At ~2 tokens per expert (64-token batched decode over 256 experts) the stage is the weight stream, and on CUDA
 * cores its cost is the code conversion and one FMA per code and token. Here one warp-wide mma.m16n8k16 takes 16
 * rows x 16 codes against 8 columns: the hi and lo fp16 terms of up to 4 tokens (the activations split per group
 * of 64 as for the tcgen05 kernels: v * 2^e = hi + lo, expert_tc.cu), so a code costs about one conversion
 * instruction whatever the chunk's token count:
 *   item       (chunk of <= 4 tokens, tile of 16 rows), one warp, walked by a persistent grid of warps; the warp
 *              streams its rows' codes over the whole K (gate and up together for gate/up)
 *   fragments  thread (g, c) = (lane / 4, lane % 4) loads 16 consecutive codes of rows g and g + 8 per group and
 *              feeds them to the 4 MMAs of the group as the k pairs {2c, 2c+1} and {2c+8, 2c+9}; the activation
 *              rows are laid out so that column n = (token n / 2, term n % 2) holds the same inputs at the same
 *              fragment slots (natural order for 8-bit codes, the nibble pairs (i, i+4) of each word for 4-bit)
 *   conversion a code pair becomes the fp16 pair (1024 + q0, 1024 + q1) by one byte permute (8-bit) or one logic
 *              op (4-bit), and one paired subtraction leaves (q0, q1): exact
 *   epilogue   per group, fp32 in registers as the reference: acc += scale * (hi + lo) * 2^-e + bias * sum(x), the
 *              tensor core's own accumulation limited to the 4 k16 steps of a group
 *   gate/up    h = silu(g) * u (ops.c:16-21) -> h3[pair][row] (fp32; split for the down projection by
 *              qe_launch_split_rows)
 *   down       y -> ybuf[pair][row], summed per token by the combine kernel in slot order (moe_layer.c:79-88)
 * The next group's codes, activations, scales and biases are loaded while this group's MMAs run.
 */
#include <atomic>

#include "qe_common.cuh"
#include "qe_kernels.h"

namespace {

constexpr int kGS = 64;
constexpr int kTok = 4;                /* tokens per chunk: the MMA's 8 columns hold their hi and lo terms */
constexpr int kWarps = 8;              /* warps per CTA (each walks its own items) */

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

/* (1024 + q0, 1024 + q1) - (1024, 1024) = (q0, q1) as an fp16 pair: exact for codes below 2^11. */
__device__ __forceinline__ uint32_t h2_sub1024(uint32_t v) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64006400u));
    return r;
}

/* The fp16 code pairs of one 32-bit word, in the order the activation layout expects:
 * 8-bit: (q0, q1), (q2, q3); 4-bit: (n0, n4), (n1, n5), (n2, n6), (n3, n7). */
template <int BITS>
__device__ __forceinline__ void code_pairs(uint32_t w, uint32_t (&p)[16 / BITS]) {
    if constexpr (BITS == 8) {
        p[0] = h2_sub1024(__byte_perm(w, 0x64646464u, 0x4140));
        p[1] = h2_sub1024(__byte_perm(w, 0x64646464u, 0x4342));
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) p[i] = h2_sub1024(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u);
    }
}

/* A thread's share of one group of a row: 16 codes (16 bytes for 8-bit, 8 bytes for 4-bit). */
template <int BITS> struct Codes;
template <> struct Codes<8> {
    uint4 v;
    __device__ __forceinline__ void load(const uint8_t *p) { v = __ldg(reinterpret_cast<const uint4 *>(p)); }
    __device__ __forceinline__ uint32_t word(int i) const { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
};
template <> struct Codes<4> {
    uint2 v;
    __device__ __forceinline__ void load(const uint8_t *p) { v = __ldg(reinterpret_cast<const uint2 *>(p)); }
    __device__ __forceinline__ uint32_t word(int i) const { return i == 0 ? v.x : v.y; }
};

/* The A fragments of MMA s (0..3) of a group from the codes of rows g (r0) and g + 8 (r8). */
template <int BITS>
__device__ __forceinline__ void a_frag(const Codes<BITS> &r0, const Codes<BITS> &r8, int s, uint32_t (&a)[4]) {
    if constexpr (BITS == 8) {      /* MMA s: bytes 4s .. 4s + 3 = word s */
        uint32_t p0[2], p8[2];
        code_pairs<8>(r0.word(s), p0);
        code_pairs<8>(r8.word(s), p8);
        a[0] = p0[0]; a[1] = p8[0]; a[2] = p0[1]; a[3] = p8[1];
    } else {                        /* MMA s: pairs 2(s%2), 2(s%2)+1 of word s/2 */
        const uint32_t w0 = r0.word(s >> 1) >> (8 * (s & 1)), w8 = r8.word(s >> 1) >> (8 * (s & 1));
        a[0] = h2_sub1024((w0 & 0x000F000Fu) | 0x64006400u);
        a[1] = h2_sub1024((w8 & 0x000F000Fu) | 0x64006400u);
        a[2] = h2_sub1024(((w0 >> 4) & 0x000F000Fu) | 0x64006400u);
        a[3] = h2_sub1024(((w8 >> 4) & 0x000F000Fu) | 0x64006400u);
    }
}

/* Everything one group step reads besides the codes: this thread's activation words (B fragments for the 4
 * MMAs), the scales and biases of its two rows, and its D-column token's unscale factor and group sum. */
struct GroupIn {
    uint4 b0, b1;          /* 8 fp16 pairs: MMA s takes (b0/b1 word 2s, 2s+1) */
    uint32_t sb0[2], sb8[2];   /* per matrix: scale | bias << 16 of rows g and g + 8 */
    float f, xs;
};

template <int BITS, bool GU>
__global__ void __launch_bounds__(kWarps * 32) gm_kernel(QeExpertArgs a, const __half *__restrict__ act, int arows,
                                                         int lda, const float *__restrict__ asum,
                                                         const float *__restrict__ ainv, int ldg_s, QeBuckets b,
                                                         int div, float *__restrict__ dst, int ldd) {
    constexpr int NM = GU ? 2 : 1;
    constexpr int GB = kGS * BITS / 8;                   /* bytes of a group in a row */
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int rows_max = GU ? max(a.gate.rows, a.sh_gate.rows) : a.hidden;
    const int ntiles = (rows_max + 15) / 16, nch = b.n_active[1];
    const int items = nch * ntiles, nwarps = gridDim.x * kWarps;
    for (int item = blockIdx.x * kWarps + (threadIdx.x >> 5); item < items; item += nwarps) {
        const int4 ch = b.chunks[item / ntiles];         /* expert, first bucket position, tokens */
        const bool sh = ch.x == a.E;
        const int e = sh ? 0 : ch.x, nt = ch.z;
        const QeQDev M0 = GU ? (sh ? a.sh_gate : a.gate) : (sh ? a.sh_down : a.down);
        const QeQDev M1 = GU ? (sh ? a.sh_up : a.up) : M0;
        const int rows = M0.rows, r0 = (item % ntiles) * 16;
        if (r0 >= rows) continue;                        /* uniform over the warp */
        const int K = M0.cols, ng = K / kGS;
        const int rg = r0 + g, rg8 = min(r0 + g + 8, rows - 1);   /* rows are a multiple of 8 */
        /* B: column g = (token g / 2, term g % 2), inputs 16c .. 16c + 15 of each group */
        const int tb = g >> 1;
        const bool bon = tb < nt;
        const int brow = bon ? b.pairs[ch.y + tb] / div : 0;
        const __half *bp = act + ((size_t)(g & 1) * arows + brow) * lda + 16 * c;
        /* D columns 2c, 2c + 1: token c's hi and lo */
        const bool don = c < nt;
        const int drow = don ? b.pairs[ch.y + c] / div : 0;
        const float *fp = ainv + (size_t)drow * ldg_s, *sp = asum + (size_t)drow * ldg_s;
        const size_t bpr = (size_t)K * BITS / 8;
        const uint8_t *c0[NM], *c8[NM];
        const uint16_t *sc[NM], *bi[NM];
#pragma unroll
        for (int mi = 0; mi < NM; mi++) {
            const QeQDev &M = mi ? M1 : M0;
            const uint8_t *base = reinterpret_cast<const uint8_t *>(M.w) + (size_t)e * rows * bpr + (size_t)c * (GB / 4);
            c0[mi] = base + (size_t)rg * bpr;
            c8[mi] = base + (size_t)rg8 * bpr;
            sc[mi] = M.scales + (size_t)e * ng * rows;   /* [expert][group][row] */
            bi[mi] = M.biases + (size_t)e * ng * rows;
        }
        auto load = [&](int gi, Codes<BITS> (&w0)[NM], Codes<BITS> (&w8)[NM], GroupIn &in) {
#pragma unroll
            for (int mi = 0; mi < NM; mi++) {
                w0[mi].load(c0[mi] + (size_t)gi * GB);
                w8[mi].load(c8[mi] + (size_t)gi * GB);
                const size_t o = (size_t)gi * rows;
                in.sb0[mi] = (uint32_t)__ldg(sc[mi] + o + rg) | ((uint32_t)__ldg(bi[mi] + o + rg) << 16);
                in.sb8[mi] = (uint32_t)__ldg(sc[mi] + o + rg8) | ((uint32_t)__ldg(bi[mi] + o + rg8) << 16);
            }
            if (bon) {
                const uint4 *q = reinterpret_cast<const uint4 *>(bp + (size_t)gi * kGS);
                in.b0 = __ldg(q);
                in.b1 = __ldg(q + 1);
            } else {
                in.b0 = in.b1 = make_uint4(0u, 0u, 0u, 0u);
            }
            in.f = don ? __ldg(fp + gi) : 0.0f;
            in.xs = don ? __ldg(sp + gi) : 0.0f;
        };
        float acc[NM][2];
#pragma unroll
        for (int mi = 0; mi < NM; mi++) acc[mi][0] = acc[mi][1] = 0.0f;
        Codes<BITS> w0[2][NM], w8[2][NM];
        GroupIn in[2];
        load(0, w0[0], w8[0], in[0]);
        /* two groups per iteration, so the double buffer is indexed by constants */
        for (int gi = 0; gi < ng; gi += 2) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (gi + u >= ng) break;
                if (gi + u + 1 < ng) load(gi + u + 1, w0[u ^ 1], w8[u ^ 1], in[u ^ 1]);
                const uint32_t bw[8] = {in[u].b0.x, in[u].b0.y, in[u].b0.z, in[u].b0.w,
                                        in[u].b1.x, in[u].b1.y, in[u].b1.z, in[u].b1.w};
#pragma unroll
                for (int mi = 0; mi < NM; mi++) {
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        uint32_t af[4];
                        a_frag<BITS>(w0[u][mi], w8[u][mi], s, af);
                        mma16816(d, af[0], af[1], af[2], af[3], bw[2 * s], bw[2 * s + 1]);
                    }
                    /* rows g and g + 8, token c: (hi + lo) * 2^-e, then scale and bias (qmat.c:43) */
                    const float p0 = __fmul_rn(__fadd_rn(d[0], d[1]), in[u].f);
                    const float p8 = __fmul_rn(__fadd_rn(d[2], d[3]), in[u].f);
                    const uint32_t s0 = in[u].sb0[mi], s8 = in[u].sb8[mi];
                    acc[mi][0] = __fadd_rn(acc[mi][0], __fmaf_rn(__uint_as_float(s0 << 16), p0,
                                                                __fmul_rn(__uint_as_float(s0 & 0xFFFF0000u), in[u].xs)));
                    acc[mi][1] = __fadd_rn(acc[mi][1], __fmaf_rn(__uint_as_float(s8 << 16), p8,
                                                                __fmul_rn(__uint_as_float(s8 & 0xFFFF0000u), in[u].xs)));
                }
            }
        }
        if (don) {
            const int pid = b.pairs[ch.y + c];
            float y0 = acc[0][0], y8 = acc[0][1];
            if constexpr (GU) {
                y0 = qe_silu_mul(acc[0][0], acc[NM - 1][0]);
                y8 = qe_silu_mul(acc[0][1], acc[NM - 1][1]);
            }
            dst[(size_t)pid * ldd + rg] = y0;
            if (r0 + g + 8 < rows) dst[(size_t)pid * ldd + r0 + g + 8] = y8;
        }
    }
}

template <int BITS, bool GU>
int launch(const QeExpertArgs *a, const __half *act, int arows, int lda, const float *asum, const float *ainv,
           int ldg_s, const QeBuckets *b, int div, float *dst, int ldd, int sms, cudaStream_t s) {
    /* resident CTAs per SM, queried once per kernel (the same on every B200): a decode step cannot afford the
     * query's host time on every launch */
    static std::atomic<int> resident{0};
    int n = resident.load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, (const void *)gm_kernel<BITS, GU>, kWarps * 32, 0) !=
                cudaSuccess || n < 1)
            n = 1;
        resident.store(n, std::memory_order_relaxed);
    }
    gm_kernel<BITS, GU><<<sms * n, kWarps * 32, 0, s>>>(*a, act, arows, lda, asum, ainv, ldg_s, *b, div, dst, ldd);
    QE_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace

/* Whether the grouped GEMVs cover this block: 4- or 8-bit codes in groups of 64, scales and biases in the
 * [expert][group][row] layout, every matrix's rows a multiple of 8 (a tile's second 8 rows are whole). */
bool qe_group_supported(const QeExpertArgs *a) {
    const int bits = a->gate.bits;
    if ((bits != 4 && bits != 8) || a->gate.group_size != kGS) return false;
    for (const QeQDev *q : {&a->gate, &a->up, &a->down, &a->sh_gate, &a->sh_up, &a->sh_down})
        if (!q->scale_t || q->rows % 8 || q->cols % kGS || q->bits != bits || q->group_size != kGS) return false;
    return true;
}

int qe_group_tokens(void) { return kTok; }

/* Gate/up + SwiGLU over the bucket's chunk list (bucket.cu with one tile per expert and chunks of kTok tokens),
 * on x split by qe_launch_tc_prep (tb->act for T rows) -> h3 [pair][ldh] (fp32). */
int qe_launch_group_gateup(const QeExpertArgs *a, const QeTcBufs *tb, int T, const QeBuckets *b, int sms, float *h3,
                           int ldh, cudaStream_t s) {
    if (!qe_group_supported(a)) QE_FAIL("grouped gate/up: unsupported shape");
    if (!b->chunks) QE_FAIL("grouped gate/up: no chunk list");
    const int ng = a->hidden / kGS;
    return a->gate.bits == 4
               ? launch<4, true>(a, tb->act, T, a->hidden, tb->actsum, tb->actinv, ng, b, a->k + 1, h3, ldh, sms, s)
               : launch<8, true>(a, tb->act, T, a->hidden, tb->actsum, tb->actinv, ng, b, a->k + 1, h3, ldh, sms, s);
}

/* Down projection over the chunk list, on h3 split by qe_launch_split_rows (tb->h3s for npairs rows) ->
 * ybuf [pair][hidden]. */
int qe_launch_group_down(const QeExpertArgs *a, const QeTcBufs *tb, int npairs, const QeBuckets *b, int sms,
                         float *ybuf, cudaStream_t s) {
    if (!qe_group_supported(a)) QE_FAIL("grouped down: unsupported shape");
    if (!b->chunks) QE_FAIL("grouped down: no chunk list");
    const int ng = tb->ldh / kGS;
    return a->gate.bits == 4
               ? launch<4, false>(a, tb->h3s, npairs, tb->ldh, tb->h3sum, tb->h3inv, ng, b, 1, ybuf, a->hidden, sms, s)
               : launch<8, false>(a, tb->h3s, npairs, tb->ldh, tb->h3sum, tb->h3inv, ng, b, 1, ybuf, a->hidden, sms,
                                  s);
}
