/* moe_oracle.c: CPU restatement of the reference's routed MoE block (TEST INFRASTRUCTURE ONLY).
 *
 * Build: oracle/Makefile, gcc -O2 -std=gnu99 -ffp-contract=off -fopenmp, no -march (x86-64 baseline has
 * no FMA, so every a*b+c below rounds twice exactly as in the reference; fmaf() is called explicitly
 * only where this file defines the order itself: the fp32 router, which has no reference counterpart).
 * Citations are file:line in hatim-mlf/moe-stream-mac.
 */
#include "moe_oracle.h"
#include "synth.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* engine/src/qmat.c:8-13 */
float or_bf16_to_f32(uint16_t h) {
    uint32_t v = (uint32_t)h << 16;
    float f;
    memcpy(&f, &v, sizeof f);
    return f;
}

/* engine/src/qgroup.c:48-53: the scalar (non-NEON) path, which is what builds on x86. Value j of the
 * group sits in w[j / (32/bits)] at bit offset (j % (32/bits)) * bits, LSB first (qgroup.h:3-9);
 * the products are summed sequentially in float. */
float or_qgroup_dot(const uint32_t *w, const float *x, int n, int bits) {
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    float s = 0.f;
    for (int j = 0; j < n; j++) s += (float)((w[j / per] >> ((j % per) * bits)) & mask) * x[j];
    return s;
}

/* engine/src/qmat.c:15-49. Validation first (y untouched on error), per-group sum of x once for all
 * rows, then per row a sequential sum over groups of scale*sum_q + bias*gsum. */
int or_qmat_matvec(const OrQMat *m, const float *x, float *y) {
    if (!m || !x || !y) return -1;
    if (m->bits != 4 && m->bits != 8) return -1;
    if (m->group_size != 32 && m->group_size != 64 && m->group_size != 128) return -1;
    if (m->rows <= 0 || m->cols <= 0) return -1;
    if (m->cols % m->group_size != 0) return -1;
    const int cols = m->cols, rows = m->rows, bits = m->bits, gs = m->group_size;
    const int ng = cols / gs, stride_w = cols * bits / 32, wpg = gs * bits / 32;
    if (ng > OR_MAX_GROUPS) return -1;
    float gsum[OR_MAX_GROUPS];
    for (int g = 0; g < ng; g++) {
        float s = 0.0f;
        for (int i = 0; i < gs; i++) s += x[g * gs + i];
        gsum[g] = s;
    }
    #pragma omp parallel for schedule(static) if (rows >= 64)
    for (int r = 0; r < rows; r++) {
        const uint32_t *wp = m->w + (size_t)r * stride_w;
        const uint16_t *sp = m->scales + (size_t)r * ng;
        const uint16_t *bp = m->biases + (size_t)r * ng;
        float sum = 0.0f;
        for (int g = 0; g < ng; g++) {
            const float sum_q = or_qgroup_dot(wp + g * wpg, x + g * gs, gs, bits);
            sum += or_bf16_to_f32(sp[g]) * sum_q + or_bf16_to_f32(bp[g]) * gsum[g];
        }
        y[r] = sum;
    }
    return 0;
}

/* engine/src/loader.c:35-41: view of expert e inside a whole [E][rows][...] expert tensor. */
OrQMat or_qmat_expert(const OrQMat *all, int e) {
    OrQMat m = *all;
    m.w += (size_t)e * all->rows * (all->cols * all->bits / 32);
    m.scales += (size_t)e * all->rows * (all->cols / all->group_size);
    m.biases += (size_t)e * all->rows * (all->cols / all->group_size);
    return m;
}

/* engine/src/ops.c:29-42: float max in index order, out = expf(x - max), double sum in index order,
 * then a float divide by (float)sum. */
void or_softmax(float *out, const float *x, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > max_val) max_val = x[i];
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
        out[i] = expf(x[i] - max_val);
        sum += out[i];
    }
    for (int i = 0; i < n; i++) out[i] /= (float)sum;
}

/* engine/src/ops.c:44-73: insertion top-k, descending; equal values keep the lower index first; at
 * capacity only a strictly larger value enters; nothing is written past idx[k-1]. */
void or_topk(int *idx, const float *x, int n, int k) {
    int count = 0;
    for (int i = 0; i < n; i++) {
        const float val = x[i];
        int pos = count;
        while (pos > 0 && x[idx[pos - 1]] < val) pos--;
        if (count == k) {
            if (x[idx[k - 1]] < val) {
                if (pos < k - 1) memmove(idx + pos + 1, idx + pos, (size_t)(k - 1 - pos) * sizeof(int));
                idx[pos] = i;
            }
        } else {
            if (pos < count) memmove(idx + pos + 1, idx + pos, (size_t)(count - pos) * sizeof(int));
            idx[pos] = i;
            count++;
        }
    }
}

/* engine/src/ops.c:16-21 */
void or_silu_mul(float *out, const float *gate, const float *up, int n) {
    for (int i = 0; i < n; i++) {
        const float g = gate[i];
        out[i] = g / (1.0f + expf(-g)) * up[i];
    }
}

/* engine/src/ops.c:23-27 */
void or_sigmoid(float *out, const float *x, int n) {
    for (int i = 0; i < n; i++) out[i] = 1.0f / (1.0f + expf(-x[i]));
}

/* The host libm expf that or_softmax calls, exported so tests can compare the device exp with it. */
float or_expf(float x) { return expf(x); }

/* expf over every float whose bit pattern lies in [lo, lo + n): the host side of the exhaustive device
 * expf comparison. */
void or_expf_bits(uint32_t lo, long long n, float *y) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < n; i++) {
        const uint32_t u = lo + (uint32_t)i;
        float x;
        memcpy(&x, &u, 4);
        y[i] = expf(x);
    }
}

/* fp32 router row (no reference counterpart: the reference's router is a quantized QMat,
 * engine/include/moe_layer.h:13). The order is defined here and reproduced by the GPU kernel:
 * consecutive chunks of OR_ROUTER_CHUNK inputs, each an fmaf chain from 0 in ascending index order,
 * and the chunk sums added in chunk order to a float total that starts at 0. */
float or_dot_f32(const float *w, const float *x, int n) {
    float total = 0.0f;
    for (int c0 = 0; c0 < n; c0 += OR_ROUTER_CHUNK) {
        const int c1 = c0 + OR_ROUTER_CHUNK < n ? c0 + OR_ROUTER_CHUNK : n;
        float acc = 0.0f;
        for (int i = c0; i < c1; i++) acc = fmaf(w[i], x[i], acc);
        total += acc;
    }
    return total;
}

int or_router_logits(const OrBlock *b, const float *x, float *logits) {
    if (b->router_f32) {
        for (int e = 0; e < b->E; e++) {
            float l = or_dot_f32(b->router_f32 + (size_t)e * b->hidden, x, b->hidden);
            if (b->router_bias) l += b->router_bias[e];
            logits[e] = l;
        }
        return 0;
    }
    return or_qmat_matvec(&b->router_q, x, logits);       /* engine/src/moe_layer.c:30 */
}

/* engine/src/moe_layer.c:31-36: softmax, top-k on the probabilities, then a float sum of the selected
 * probabilities in top-k order and score_i = p_i / sum. */
int or_route_from_logits(const float *logits, int E, int k, float *probs, int *idx, float *score) {
    if (k < 1 || k > OR_MAX_TOPK || k > E) return -1;
    or_softmax(probs, logits, E);
    or_topk(idx, probs, E, k);
    float sum = 0.0f;
    for (int i = 0; i < k; i++) sum += probs[idx[i]];
    for (int i = 0; i < k; i++) score[i] = probs[idx[i]] / sum;
    return 0;
}

/* engine/src/moe_layer.c:20-26 */
static int mlp(const OrQMat *gate, const OrQMat *up, const OrQMat *down, const float *x, float *y,
               float *h1, float *h2, float *h3) {
    if (or_qmat_matvec(gate, x, h1)) return -1;
    if (or_qmat_matvec(up, x, h2)) return -1;
    or_silu_mul(h3, h1, h2, gate->rows);
    if (or_qmat_matvec(down, h3, y)) return -1;
    return 0;
}

/* engine/src/moe_layer.c:66-89, with the experts already resident (no fetch, no trace). */
int or_moe_step(const OrBlock *b, const float *x, float *out, int *idx_out, float *score_out) {
    if (b->top_k < 1 || b->top_k > OR_MAX_TOPK) return -1;
    const int m = b->inter > b->sh_inter ? b->inter : b->sh_inter;
    float *buf = malloc(sizeof(float) * (size_t)(2 * b->E + 3 * m + b->hidden + 1));
    if (!buf) return -1;
    float *logits = buf, *probs = logits + b->E, *h1 = probs + b->E, *h2 = h1 + m, *h3 = h2 + m,
          *ye = h3 + m, *gsh = ye + b->hidden;
    int idx[OR_MAX_TOPK];
    float score[OR_MAX_TOPK];
    int rc = -1;
    if (or_router_logits(b, x, logits) || or_route_from_logits(logits, b->E, b->top_k, probs, idx, score))
        goto done;
    memset(out, 0, sizeof(float) * (size_t)b->hidden);
    for (int i = 0; i < b->top_k; i++) {
        const OrQMat g = or_qmat_expert(&b->gate, idx[i]), u = or_qmat_expert(&b->up, idx[i]),
                     d = or_qmat_expert(&b->down, idx[i]);
        if (mlp(&g, &u, &d, x, ye, h1, h2, h3)) goto done;
        for (int j = 0; j < b->hidden; j++) out[j] += score[i] * ye[j];
    }
    if (mlp(&b->sh_gate, &b->sh_up, &b->sh_down, x, ye, h1, h2, h3)) goto done;
    if (b->sh_gate_f32) gsh[0] = or_dot_f32(b->sh_gate_f32, x, b->hidden);
    else if (or_qmat_matvec(&b->sh_router_q, x, gsh)) goto done;
    const float sg = 1.0f / (1.0f + expf(-gsh[0]));
    for (int j = 0; j < b->hidden; j++) out[j] += sg * ye[j];
    if (idx_out) memcpy(idx_out, idx, sizeof(int) * (size_t)b->top_k);
    if (score_out) memcpy(score_out, score, sizeof(float) * (size_t)b->top_k);
    rc = 0;
done:
    free(buf);
    return rc;
}

/* One expert's SwiGLU MLP (moe_layer.c:20-26): e in [0, E) a routed expert, e = -1 the shared expert. */
int or_expert_mlp(const OrBlock *b, int e, const float *x, float *y) {
    if (e < -1 || e >= b->E) return -1;
    const int m = b->inter > b->sh_inter ? b->inter : b->sh_inter;
    float *buf = malloc(sizeof(float) * (size_t)(3 * m));
    if (!buf) return -1;
    int rc;
    if (e < 0) {
        rc = mlp(&b->sh_gate, &b->sh_up, &b->sh_down, x, y, buf, buf + m, buf + 2 * m);
    } else {
        const OrQMat g = or_qmat_expert(&b->gate, e), u = or_qmat_expert(&b->up, e), d = or_qmat_expert(&b->down, e);
        rc = mlp(&g, &u, &d, x, y, buf, buf + m, buf + 2 * m);
    }
    free(buf);
    return rc;
}

/* The shared-expert gate logit (moe_layer.c:85-87): w_sg . x in fp32 mode, else the shared_expert_gate QMat. */
int or_shared_gate_logit(const OrBlock *b, const float *x, float *g) {
    if (b->sh_gate_f32) {
        g[0] = or_dot_f32(b->sh_gate_f32, x, b->hidden);
        return 0;
    }
    return or_qmat_matvec(&b->sh_router_q, x, g);
}

/* T independent tokens (the reference has no batched prefill, docs/C_ENGINE.md:81: prefill is T calls
 * of moe_layer_step). Tokens run in parallel here; each token's arithmetic is unchanged. */
int or_moe_forward(const OrBlock *b, int T, const float *x, float *out, int *idx, float *score) {
    int failed = 0;
    #pragma omp parallel for schedule(dynamic, 1) reduction(| : failed)
    for (int t = 0; t < T; t++)
        failed |= or_moe_step(b, x + (size_t)t * b->hidden, out + (size_t)t * b->hidden,
                              idx ? idx + (size_t)t * b->top_k : NULL,
                              score ? score + (size_t)t * b->top_k : NULL) != 0;
    return failed ? -1 : 0;
}

int or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* ---- synthetic blocks (same generator as the GPU library: csrc/synth.h) ---- */

static OrQMat synth_qmat(uint64_t seed, uint32_t block, uint32_t stream, int n, int rows, int cols, int bits,
                         int gs) {
    const size_t wpr = (size_t)cols * bits / 32, ng = (size_t)cols / gs;
    uint32_t *w = malloc(sizeof(uint32_t) * n * rows * wpr);
    uint16_t *s = malloc(sizeof(uint16_t) * n * rows * ng), *bb = malloc(sizeof(uint16_t) * n * rows * ng);
    const float sc = syn_scale_c(bits), nh = syn_neg_half_range(bits);
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)(n * rows * wpr); i++) w[i] = syn_code_word(seed, block, stream, (uint64_t)i);
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)(n * rows * ng); i++)
        syn_scale_bias(seed, block, stream, (uint64_t)i, sc, nh, &s[i], &bb[i]);
    OrQMat m = { w, s, bb, rows, cols, bits, gs };
    return m;
}

static float *synth_normal_vec(uint64_t seed, uint32_t block, uint32_t stream, size_t n, double sigma) {
    float *v = malloc(sizeof(float) * n);
    const float c = syn_sigma_c(sigma);
    for (size_t i = 0; i < n; i++) v[i] = syn_normal(syn_hash(seed, block, stream, i), c);
    return v;
}

OrBlock *or_synth_block(const OrSynthCfg *c, uint64_t seed, uint32_t block, const float *router_bias) {
    OrBlock *b = calloc(1, sizeof *b);
    if (!b) return NULL;
    b->hidden = c->hidden; b->E = c->E; b->top_k = c->top_k; b->inter = c->inter; b->sh_inter = c->sh_inter;
    const int H = c->hidden, bits = c->bits, gs = c->group_size;
    b->gate = synth_qmat(seed, block, SYN_GATE, c->E, c->inter, H, bits, gs);
    b->up = synth_qmat(seed, block, SYN_UP, c->E, c->inter, H, bits, gs);
    b->down = synth_qmat(seed, block, SYN_DOWN, c->E, H, c->inter, bits, gs);
    b->sh_gate = synth_qmat(seed, block, SYN_SH_GATE, 1, c->sh_inter, H, bits, gs);
    b->sh_up = synth_qmat(seed, block, SYN_SH_UP, 1, c->sh_inter, H, bits, gs);
    b->sh_down = synth_qmat(seed, block, SYN_SH_DOWN, 1, H, c->sh_inter, bits, gs);
    if (c->quant_router) {
        b->router_q = synth_qmat(seed, block, SYN_ROUTER, 1, c->E, H, 8, gs);
        b->sh_router_q = synth_qmat(seed, block, SYN_SHGATE, 1, 1, H, 8, gs);
    } else {
        b->router_f32 = synth_normal_vec(seed, block, SYN_ROUTER, (size_t)c->E * H, 0.02);
        b->sh_gate_f32 = synth_normal_vec(seed, block, SYN_SHGATE, (size_t)H, 0.02);
        if (router_bias) {
            float *rb = malloc(sizeof(float) * c->E);
            memcpy(rb, router_bias, sizeof(float) * c->E);
            b->router_bias = rb;
        }
    }
    return b;
}

static void free_q(OrQMat *m) { free((void *)m->w); free((void *)m->scales); free((void *)m->biases); }

void or_free_block(OrBlock *b) {
    if (!b) return;
    free_q(&b->gate); free_q(&b->up); free_q(&b->down);
    free_q(&b->sh_gate); free_q(&b->sh_up); free_q(&b->sh_down);
    free_q(&b->router_q); free_q(&b->sh_router_q);
    free((void *)b->router_f32); free((void *)b->router_bias); free((void *)b->sh_gate_f32);
    free(b);
}

void or_synth_x(float *x, int T, int hidden, uint64_t seed, uint32_t block) {
    const float c = syn_sigma_c(1.0);
    for (size_t i = 0; i < (size_t)T * hidden; i++) x[i] = syn_normal(syn_hash(seed, block, SYN_X, i), c);
}
