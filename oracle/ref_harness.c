/* ref_harness.c: drives the UNMODIFIED reference sources, compiled from where they lie in the reference
 * checkout by oracle/Makefile into oracle/_ref/libqref.so (TEST INFRASTRUCTURE ONLY: it pins the
 * restatement in moe_oracle.c and serves as the reference arm of the CPU baseline).
 *
 * Mode R: the reference's own moe_layer_step (engine/src/moe_layer.c:66-89) on a safetensors checkpoint
 *         directory, with experts pread from disk (expert_store.c:54-61) exactly as the engine runs them.
 *         The opening sequence follows what engine/src/model.c:52-82 (load_moe) does for one layer.
 * Mode B: the benchmark configurations' fp32 router and fp32 shared-expert gate have no reference
 *         counterpart (the reference router is a quantized QMat, moe_layer.h:13), so this file restates
 *         moe_layer_step's control flow around the reference's own qmat_matvec, op_softmax, op_topk and
 *         op_silu_mul, with the experts held in RAM (loader.c:35-41 expert views). Only the fp32 dot
 *         products are harness code; their order matches or_dot_f32 in moe_oracle.c.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "expert_store.h"
#include "k3_st.h"
#include "loader.h"
#include "moe_layer.h"
#include "ops.h"
#include "qmat.h"
#include "moe_oracle.h"
#ifdef _OPENMP
#include <omp.h>
#endif

static QMat q_of(const OrQMat *m) {
    QMat q = { m->w, m->scales, m->biases, m->rows, m->cols, m->bits, m->group_size };
    return q;
}

/* Same order as or_dot_f32 (moe_oracle.c): 64-input fmaf chains, chunk sums added in order. */
static float harness_dot_f32(const float *w, const float *x, int n) {
    float total = 0.0f;
    for (int c0 = 0; c0 < n; c0 += 64) {
        const int c1 = c0 + 64 < n ? c0 + 64 : n;
        float acc = 0.0f;
        for (int i = c0; i < c1; i++) acc = fmaf(w[i], x[i], acc);
        total += acc;
    }
    return total;
}

static int mlp(const QMat *gate, const QMat *up, const QMat *down, const float *x, float *y, float *h1,
               float *h2, float *h3) {
    if (qmat_matvec(gate, x, h1)) return -1;
    if (qmat_matvec(up, x, h2)) return -1;
    op_silu_mul(h3, h1, h2, gate->rows);
    if (qmat_matvec(down, h3, y)) return -1;
    return 0;
}

/* Mode B, one token. scratch as MOE_SCRATCH_FLOATS (moe_layer.h:24). */
int ref_b_step(const OrBlock *b, const float *x, float *out, int *idx_out, float *score_out, float *scratch) {
    if (b->top_k < 1 || b->top_k > MOE_MAX_TOPK) return -1;
    const int m = b->inter > b->sh_inter ? b->inter : b->sh_inter;
    float *logits = scratch, *probs = logits + b->E, *h1 = probs + b->E, *h2 = h1 + m, *h3 = h2 + m,
          *ye = h3 + m;
    if (b->router_f32) {
        for (int e = 0; e < b->E; e++) {
            float l = harness_dot_f32(b->router_f32 + (size_t)e * b->hidden, x, b->hidden);
            if (b->router_bias) l += b->router_bias[e];
            logits[e] = l;
        }
    } else {
        const QMat r = q_of(&b->router_q);
        if (qmat_matvec(&r, x, logits)) return -1;
    }
    op_softmax(probs, logits, b->E);
    int idx[MOE_MAX_TOPK];
    float score[MOE_MAX_TOPK];
    op_topk(idx, probs, b->E, b->top_k);
    float sum = 0.0f;
    for (int i = 0; i < b->top_k; i++) sum += probs[idx[i]];
    for (int i = 0; i < b->top_k; i++) score[i] = probs[idx[i]] / sum;
    const QMat G = q_of(&b->gate), U = q_of(&b->up), D = q_of(&b->down);
    memset(out, 0, sizeof(float) * (size_t)b->hidden);
    for (int i = 0; i < b->top_k; i++) {
        const QMat g = qmat_expert(&G, idx[i]), u = qmat_expert(&U, idx[i]), d = qmat_expert(&D, idx[i]);
        if (mlp(&g, &u, &d, x, ye, h1, h2, h3)) return -1;
        for (int j = 0; j < b->hidden; j++) out[j] += score[i] * ye[j];
    }
    const QMat sg_ = q_of(&b->sh_gate), su = q_of(&b->sh_up), sd = q_of(&b->sh_down);
    if (mlp(&sg_, &su, &sd, x, ye, h1, h2, h3)) return -1;
    float gsh;
    if (b->sh_gate_f32) {
        gsh = harness_dot_f32(b->sh_gate_f32, x, b->hidden);
    } else {
        const QMat r = q_of(&b->sh_router_q);
        if (qmat_matvec(&r, x, &gsh)) return -1;
    }
    const float sg = 1.0f / (1.0f + expf(-gsh));
    for (int j = 0; j < b->hidden; j++) out[j] += sg * ye[j];
    if (idx_out) memcpy(idx_out, idx, sizeof(int) * (size_t)b->top_k);
    if (score_out) memcpy(score_out, score, sizeof(float) * (size_t)b->top_k);
    return 0;
}

/* Mode B over T tokens, one after the other as the engine's prefill does (qchat.py:64-67); the
 * parallelism is the reference's own OpenMP inside qmat_matvec (qmat.c:35). */
int ref_b_forward(const OrBlock *b, int T, const float *x, float *out, int *idx, float *score) {
    const int m = b->inter > b->sh_inter ? b->inter : b->sh_inter;
    float *scratch = malloc(sizeof(float) * (size_t)(2 * b->E + 3 * m + b->hidden + 1));
    if (!scratch) return -1;
    int rc = 0;
    for (int t = 0; t < T && rc == 0; t++)
        rc = ref_b_step(b, x + (size_t)t * b->hidden, out + (size_t)t * b->hidden,
                        idx ? idx + (size_t)t * b->top_k : NULL, score ? score + (size_t)t * b->top_k : NULL,
                        scratch);
    free(scratch);
    return rc;
}

/* ---- Mode R: unmodified moe_layer_step on a checkpoint directory ---- */

typedef struct {
    K3St st;
    MoeWeights w;
    float *scratch;
} RefR;

void *ref_r_open(const char *dir, const char *prefix, int hidden, int top_k, int inter, int sh_inter, int gs) {
    RefR *h = calloc(1, sizeof *h);
    if (!h) return NULL;
    if (k3_st_open(&h->st, dir)) { free(h); return NULL; }
    MoeWeights *w = &h->w;
    char name[512];
    const char *ex[3] = { "switch_mlp.gate_proj", "switch_mlp.up_proj", "switch_mlp.down_proj" };
    ExpertTensor *et[3] = { &w->gate, &w->up, &w->down };
    ExpertBuf *eb[3] = { w->gbuf, w->ubuf, w->dbuf };
    for (int i = 0; i < 3; i++) {
        snprintf(name, sizeof name, "%s.%s", prefix, ex[i]);
        if (expert_tensor_open(et[i], &h->st, name, gs)) return NULL;
        for (int k = 0; k < top_k && k < MOE_MAX_TOPK; k++)
            if (expert_buf_alloc(&eb[i][k], et[i])) return NULL;
    }
    const char *parts[5] = { "gate", "shared_expert.gate_proj", "shared_expert.up_proj", "shared_expert.down_proj",
                             "shared_expert_gate" };
    QMat *dst[5] = { &w->router, &w->sh_gate, &w->sh_up, &w->sh_down, &w->sh_router };
    for (int i = 0; i < 5; i++) {
        snprintf(name, sizeof name, "%s.%s", prefix, parts[i]);
        if (load_qmat(&h->st, name, gs, dst[i], NULL)) return NULL;
    }
    w->hidden = hidden; w->E = w->gate.E; w->top_k = top_k; w->inter = inter; w->sh_inter = sh_inter;
    h->scratch = malloc(sizeof(float) * (size_t)MOE_SCRATCH_FLOATS(w));
    return h->scratch ? h : NULL;
}

int ref_r_step(void *hp, const float *x, float *out) {
    RefR *h = hp;
    return moe_layer_step(out, x, &h->w, h->scratch);
}

/* The reference's top_k bound check (moe_layer.c:67): a block with top_k beyond MOE_MAX_TOPK is refused. */
int ref_r_step_with_topk(void *hp, int top_k, const float *x, float *out) {
    RefR *h = hp;
    MoeWeights w = h->w;
    w.top_k = top_k;
    return moe_layer_step(out, x, &w, h->scratch);
}

int ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

double ref_expert_gb_read(void) { return expert_bytes_read() / 1e9; }
