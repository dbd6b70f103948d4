/* route_dev.cuh: device functions of the router and of the softmax/top-k/renormalisation, shared by the
 * routing kernels (route.cu) and the fused decode kernel (decode.cu). Bit-exact with the reference:
 * engine/src/moe_layer.c:29-37 (route), engine/src/ops.c:29-73 (op_softmax, op_topk); the fp32 router's
 * dot-product order is defined once and followed by the CPU checker (or_dot_f32 in oracle/moe_oracle.c).
 */
#ifndef QE_ROUTE_DEV_CUH
#define QE_ROUTE_DEV_CUH
#include "qe_common.cuh"

namespace {

constexpr int kRouterChunk = 64;       /* fp32 router chunk length (or_dot_f32) */
constexpr int kRouterLaneChunks = 4;   /* hidden <= 32 * 4 * 64 = 8192 */
constexpr int kRouterGemvTokens = 8;

/* Decode / small batch: one warp per router row (E routed rows + the shared gate row). Lane c owns
 * chunks c, c+32, ...; each chunk is an fmaf chain per token; lane 0..nt-1 then add the chunk sums in
 * chunk order. vec (W, x 16-byte aligned, H % 4 == 0): a lane requests its whole 64-float weight chunk
 * with 16-byte loads before the chain starts. */
__device__ __forceinline__ void router_row_f32(const float *__restrict__ W, const float *__restrict__ bias,
                                               const float *__restrict__ x, int T, int H, int E, int row,
                                               float *__restrict__ logits, int vec) {
    const int lane = threadIdx.x & 31;
    const float *w = W + (size_t)row * H;
    const int nch = (H + kRouterChunk - 1) / kRouterChunk;
    const int ld = E + 1;
    for (int t0 = 0; t0 < T; t0 += kRouterGemvTokens) {
        const int nt = min(kRouterGemvTokens, T - t0);
        float acc[kRouterLaneChunks][kRouterGemvTokens];
#pragma unroll
        for (int cc = 0; cc < kRouterLaneChunks; cc++) {
#pragma unroll
            for (int t = 0; t < kRouterGemvTokens; t++) acc[cc][t] = 0.0f;
            const int c = lane + 32 * cc;
            if (c < nch && vec && (c + 1) * kRouterChunk <= H) {
                const float4 *w4 = reinterpret_cast<const float4 *>(w + (size_t)c * kRouterChunk);
                float4 wv[kRouterChunk / 4];
#pragma unroll
                for (int q = 0; q < kRouterChunk / 4; q++) wv[q] = __ldg(w4 + q);
#pragma unroll
                for (int t = 0; t < kRouterGemvTokens; t++) {
                    if (t >= nt) break;
                    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)(t0 + t) * H + (size_t)c * kRouterChunk);
                    float a = 0.0f;
#pragma unroll
                    for (int q = 0; q < kRouterChunk / 4; q++) {
                        const float4 xv = __ldg(x4 + q);
                        a = __fmaf_rn(wv[q].x, xv.x, a);
                        a = __fmaf_rn(wv[q].y, xv.y, a);
                        a = __fmaf_rn(wv[q].z, xv.z, a);
                        a = __fmaf_rn(wv[q].w, xv.w, a);
                    }
                    acc[cc][t] = a;
                }
            } else if (c < nch) {
                const int i0 = c * kRouterChunk, i1 = min(i0 + kRouterChunk, H);
                for (int i = i0; i < i1; i++) {
                    const float wv = __ldg(w + i);
#pragma unroll
                    for (int t = 0; t < kRouterGemvTokens; t++)
                        if (t < nt) acc[cc][t] = __fmaf_rn(wv, __ldg(x + (size_t)(t0 + t) * H + i), acc[cc][t]);
                }
            }
        }
        float total[kRouterGemvTokens];
#pragma unroll
        for (int t = 0; t < kRouterGemvTokens; t++) total[t] = 0.0f;
#pragma unroll
        for (int cc = 0; cc < kRouterLaneChunks; cc++) {
            if (cc * 32 >= nch) break;
            for (int src = 0; src < 32; src++) {
                if (cc * 32 + src >= nch) break;
#pragma unroll
                for (int t = 0; t < kRouterGemvTokens; t++) {
                    if (t >= nt) break;   /* nt is the same for the whole warp: no shuffle for absent tokens */
                    const float v = __shfl_sync(QE_FULL, acc[cc][t], src);
                    total[t] = __fadd_rn(total[t], v);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kRouterGemvTokens; t++) {
            if (lane == t && t < nt) {
                float l = total[t];
                if (bias && row < E) l = __fadd_rn(l, bias[row]);
                logits[(size_t)(t0 + t) * ld + row] = l;
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------------
 * Softmax + top-k + renormalisation: one warp per token, bit-exact with ops.c:29-73 + moe_layer.c:31-36.
 *   max     : order-independent for non-NaN input (a NaN anywhere takes the sequential path).
 *   e_i     : qe_expf(x_i - max), identical to the host expf.
 *   sum     : ops.c adds the e_i in DOUBLE in index order. The warp adds them pairwise in double and
 *             proves that rounding to float gives the same value: the sequential and the pairwise sums
 *             each lie within (n-1)u*S of the exact sum (u = 2^-53, all terms positive), so if the
 *             interval [S_pair - B, S_pair + B], B = (2n+8) u S_pair, lies strictly inside the rounding
 *             interval of f = (float)S_pair, then (float)S_seq == f. Otherwise (probability ~ n*2^-29)
 *             lane 0 repeats the sum sequentially.
 *   p_i     : e_i / (float)sum, IEEE division.
 *   top-k   : op_topk's insertion sort keeps values in descending order and equal values in index
 *             order, and at capacity admits only a strictly larger value; for non-NaN input that is the
 *             first k of the order (p desc, index asc), found here by k rounds of warp arg-max.
 *   score_i : p_sel_i / (float sum of p_sel in top-k order).
 * ------------------------------------------------------------------------------------------------- */
constexpr int kMaxEPL = 16; /* E <= 512 */

__device__ __noinline__ void route_token_sequential(const float *lg, int E, int k, float *probs_s, int *idx_s, int32_t *idx,
                                       float *score, float *probs_out) {
    /* ops.c:29-42 literally */
    float max_val = lg[0];
    for (int i = 1; i < E; i++)
        if (lg[i] > max_val) max_val = lg[i];
    double sum = 0.0;
    for (int i = 0; i < E; i++) {
        probs_s[i] = qe_expf(__fsub_rn(lg[i], max_val));
        sum = __dadd_rn(sum, (double)probs_s[i]);
    }
    const float sf = __double2float_rn(sum);
    for (int i = 0; i < E; i++) probs_s[i] = __fdiv_rn(probs_s[i], sf);
    /* ops.c:44-73 literally */
    int count = 0;
    for (int i = 0; i < E; i++) {
        const float val = probs_s[i];
        int pos = count;
        while (pos > 0 && probs_s[idx_s[pos - 1]] < val) pos--;
        if (count == k) {
            if (probs_s[idx_s[k - 1]] < val) {
                for (int j = k - 1; j > pos; j--) idx_s[j] = idx_s[j - 1];
                idx_s[pos] = i;
            }
        } else {
            for (int j = count; j > pos; j--) idx_s[j] = idx_s[j - 1];
            idx_s[pos] = i;
            count++;
        }
    }
    float s = 0.0f;
    for (int i = 0; i < k; i++) s = __fadd_rn(s, probs_s[idx_s[i]]);
    for (int i = 0; i < k; i++) {
        idx[i] = idx_s[i];
        score[i] = __fdiv_rn(probs_s[idx_s[i]], s);
    }
    if (probs_out)
        for (int i = 0; i < E; i++) probs_out[i] = probs_s[i];
}

template <int EPL>
__device__ __forceinline__ void route_topk_warp_t(const float *__restrict__ lg, int t, int E, int k, float *probs_s,
                                                  int *idx_s, int32_t *__restrict__ idx_out,
                                                  float *__restrict__ score_out, float *__restrict__ probs_out) {
    /* lane holds experts lane + 32*i, i < EPL; slots past E hold -inf (exp 0, never selected before a valid
     * expert: equal values keep the lower index). The per-slot loops carry no conditions, so the lane's
     * exponentials and divisions run as independent chains. */
    const int lane = threadIdx.x & 31;
    float v[EPL];
    bool has_nan = false;
    float mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        v[i] = e < E ? lg[e] : -__int_as_float(0x7f800000);
        has_nan |= (v[i] != v[i]);
        mx = fmaxf(mx, v[i]);
    }
    has_nan = __any_sync(QE_FULL, has_nan);
    if (has_nan) {
        if (lane == 0)
            route_token_sequential(lg, E, k, probs_s, idx_s, idx_out + (size_t)t * k, score_out + (size_t)t * k,
                                   probs_out ? probs_out + (size_t)t * E : nullptr);
        return;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(QE_FULL, mx, o));

#pragma unroll
    for (int i = 0; i < EPL; i++) v[i] = qe_expf(__fsub_rn(v[i], mx));
    double part = 0.0;   /* slots past E add +0.0: no change */
#pragma unroll
    for (int i = 0; i < EPL; i++) part = __dadd_rn(part, (double)v[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(QE_FULL, part, o));
    float sf = __double2float_rn(part);
    {
        const double B = (double)(2 * E + 8) * 0x1p-53 * part;
        const float up = nextafterf(sf, __int_as_float(0x7f800000)), dn = nextafterf(sf, 0.0f);
        const double mid_hi = ((double)sf + (double)up) * 0.5, mid_lo = ((double)sf + (double)dn) * 0.5;
        const bool safe = (part - B > mid_lo) && (part + B < mid_hi);
        if (!safe) { /* uniform across the warp: every lane holds the same part */
#pragma unroll
            for (int i = 0; i < EPL; i++) {
                const int e = lane + 32 * i;
                if (e < E) probs_s[e] = v[i];
            }
            __syncwarp();
            double seq = 0.0;
            if (lane == 0)
                for (int e = 0; e < E; e++) seq = __dadd_rn(seq, (double)probs_s[e]);
            seq = __shfl_sync(QE_FULL, seq, 0);
            sf = __double2float_rn(seq);
            __syncwarp();
        }
    }
    unsigned used = 0;
#pragma unroll
    for (int i = 0; i < EPL; i++) v[i] = __fdiv_rn(v[i], sf);
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        if (e < E) {
            if (probs_out) probs_out[(size_t)t * E + e] = v[i];
        } else {
            used |= 1u << i; /* not a candidate */
        }
    }
    float psel = 0.0f, ssum = 0.0f;
    int isel = 0;
    for (int r = 0; r < k; r++) {
        float bv = -__int_as_float(0x7f800000);
        int bi = 0x7fffffff, bslot = -1;
#pragma unroll
        for (int i = 0; i < EPL; i++) {
            if (!(used >> i & 1u) && (bslot < 0 || v[i] > bv)) { /* ascending i = ascending index */
                bv = v[i];
                bi = lane + 32 * i;
                bslot = i;
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(QE_FULL, bv, o);
            const int oi = __shfl_xor_sync(QE_FULL, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bslot >= 0 && bi == lane + 32 * bslot) used |= 1u << bslot;
        ssum = __fadd_rn(ssum, bv);
        if (lane == r) {
            psel = bv;
            isel = bi;
        }
    }
    if (lane < k) {
        idx_out[(size_t)t * k + lane] = isel;
        score_out[(size_t)t * k + lane] = __fdiv_rn(psel, ssum);
    }
}

/* Token t (one warp): lg = its logits, probs_s/idx_s = 2*E floats of this warp's shared memory; writes
 * idx_out[t*k ..], score_out[t*k ..] and, when probs_out is given, probs_out[t*E ..]. E <= 32*kMaxEPL. */
__device__ __forceinline__ void route_topk_warp(const float *__restrict__ lg, int t, int E, int k, float *probs_s,
                                                int *idx_s, int32_t *__restrict__ idx_out,
                                                float *__restrict__ score_out, float *__restrict__ probs_out) {
    const int epl = (E + 31) / 32;
    if (epl <= 1) route_topk_warp_t<1>(lg, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
    else if (epl <= 2) route_topk_warp_t<2>(lg, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
    else if (epl <= 4) route_topk_warp_t<4>(lg, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
    else if (epl <= 8) route_topk_warp_t<8>(lg, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
    else route_topk_warp_t<16>(lg, t, E, k, probs_s, idx_s, idx_out, score_out, probs_out);
}

}  // namespace

#endif
