/* moe_oracle.h: CPU restatement of the reference C engine's routed MoE block (TEST INFRASTRUCTURE ONLY).
 *
 * This is the checker the CUDA path is compared against. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product library never links or calls it.
 *
 * Each function restates one function of hatim-mlf/moe-stream-mac (paths relative to that project) with
 * the same float operation order, so that a gcc build without -march/-ffast-math (no FMA contraction,
 * x86 scalar qgroup_dot path) is bit-identical to the reference compiled the same way. The
 * restatement is pinned two ways by tests/test_oracle_golden.py: against the reference's committed
 * fixtures (engine/tests/fixtures) and against the reference sources compiled into oracle/_ref.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stdint.h>

#define OR_MAX_TOPK 16              /* engine/include/moe_layer.h:10 */
#define OR_MAX_GROUPS 4096          /* engine/src/qmat.c:4 */
#define OR_ROUTER_CHUNK 64          /* fp32 router: fmaf chains over 64 inputs, chunks added in order */

/* engine/include/qmat.h:17-25 */
typedef struct {
    const uint32_t *w;
    const uint16_t *scales;
    const uint16_t *biases;
    int rows, cols, bits, group_size;
} OrQMat;

/* engine/include/moe_layer.h:12-21, with the routed experts held in RAM as whole [E][rows][...] tensors
 * (engine/src/loader.c:16-41 load_qmat + qmat_expert) instead of pread buffers, and two fp32 options the
 * benchmark configurations need: an fp32 router [E][hidden] (+ optional per-expert logit bias) and an
 * fp32 shared-expert gate vector [hidden]. */
typedef struct {
    int hidden, E, top_k, inter, sh_inter;
    const float *router_f32;       /* [E][hidden] or NULL -> router_q            */
    const float *router_bias;      /* [E] added to the fp32 logits, or NULL       */
    OrQMat router_q;
    OrQMat gate, up, down;         /* 3-D: rows/cols of ONE expert; w/scales/biases cover all E */
    OrQMat sh_gate, sh_up, sh_down;
    const float *sh_gate_f32;      /* [hidden] or NULL -> sh_router_q             */
    OrQMat sh_router_q;
} OrBlock;

float or_bf16_to_f32(uint16_t h);
float or_qgroup_dot(const uint32_t *w, const float *x, int n, int bits);
int or_qmat_matvec(const OrQMat *m, const float *x, float *y);
OrQMat or_qmat_expert(const OrQMat *all, int e);
void or_softmax(float *out, const float *x, int n);
void or_topk(int *idx, const float *x, int n, int k);
void or_silu_mul(float *out, const float *gate, const float *up, int n);
void or_sigmoid(float *out, const float *x, int n);
float or_expf(float x);
void or_expf_bits(uint32_t lo, long long n, float *y);
float or_dot_f32(const float *w, const float *x, int n);
int or_router_logits(const OrBlock *b, const float *x, float *logits);
int or_route_from_logits(const float *logits, int E, int k, float *probs, int *idx, float *score);
int or_moe_step(const OrBlock *b, const float *x, float *out, int *idx, float *score);
int or_moe_forward(const OrBlock *b, int T, const float *x, float *out, int *idx, float *score);
int or_expert_mlp(const OrBlock *b, int e, const float *x, float *y);
int or_shared_gate_logit(const OrBlock *b, const float *x, float *g);

/* Synthetic block generation (moe-stream-mac_b200/csrc/synth.h), for tests and the CPU baseline. */
typedef struct {
    int hidden, E, top_k, inter, sh_inter, bits, group_size;
    int quant_router;              /* 0: fp32 router + fp32 shared gate; 1: 8-bit quantized router + sh gate */
} OrSynthCfg;
OrBlock *or_synth_block(const OrSynthCfg *c, uint64_t seed, uint32_t block, const float *router_bias);
void or_free_block(OrBlock *b);
void or_synth_x(float *x, int T, int hidden, uint64_t seed, uint32_t block);
int or_set_threads(int n);

#endif
