/* qe_engine.h: the whole-model C ABI of libqengine_b200, under the names and signatures of the reference
 * engine's front-end API (engine/include/qengine.h:9-23, implemented in engine/src/qengine.c:12-47), so that
 * a ctypes front end bound to that API (engine/cli/qchat.py:34-62, class Engine) drives this library
 * unchanged once it loads libqengine_b200.so instead of libqengine.
 *
 * One qwen3_5_moe MLX checkpoint, one token per qe_forward call (model.c:148-157): the embedding row, per
 * layer RMSNorm -> Gated DeltaNet or gated full attention -> residual -> RMSNorm -> routed MoE block ->
 * residual (model.c:135-146), the final RMSNorm and the LM head. The routed MoE blocks run on the GPU
 * (one qe_moe handle per layer, experts resident in HBM, include/qe_moe.h). The rest of the layer (the
 * "trunk") runs on the same GPU by default: its tensors are copied to HBM at qe_load and a token's whole step
 * stays on the device, the logits being the only copy back. With QE_TRUNK=host in the environment at qe_load,
 * the trunk runs on the host in fp32 on qe_set_threads threads instead, reading the checkpoint's memory
 * mappings. Conventions as the reference's: NULL from qe_load with the reason on stderr; 0 ok, -1 error,
 * -2 context full. qe_set_threads, qe_expert_gb_read, qe_expert_read_seconds and qe_peak_rss_gb (the rest of
 * qengine.h) are declared in qe_moe.h.
 */
#ifndef QE_ENGINE_H
#define QE_ENGINE_H
#include "qe_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct QeModel QeModel;

/* Load <dir>/config.json (strictly: every field the model needs, model_type qwen3_5_moe*, affine
 * quantization, default RoPE) and every *.safetensors shard of dir. max_len = context length in tokens
 * (>= 1). The MoE blocks go to CUDA device QE_DEVICE (environment, default 0). NULL on failure.
 * Replaces qe_load (qengine.c:12-17). */
QeModel *qe_load(const char *dir, int max_len);
/* Releases the handle, its GPU blocks and its mappings (the reference keeps weights until exit). */
void qe_free(QeModel *m);
/* Forget the sequence: recurrent states and KV caches cleared, position 0 (qengine.c:21). */
void qe_reset(QeModel *m);
/* Feed one token at the next position; logits receives qe_vocab(m) floats. 0 ok, -1 error (a bad token id,
 * a failed GPU call), -2 context full (call qe_reset). Replaces qe_forward (qengine.c:23-29). */
int qe_forward(QeModel *m, int token, float *logits);
int qe_vocab(const QeModel *m);
int qe_position(const QeModel *m);   /* tokens fed since the last reset */
int qe_max_len(const QeModel *m);

/* The trunk's host ops, exported for the fixture tests (the reference's own fixtures pin them:
 * engine/tests/test_ops.c, test_gdn.c). Same contracts as engine/include/ops.h and gdn.h. */
void qe_trunk_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void qe_trunk_rope(float *x, int n_heads, int head_dim, int rot_dims, int pos, float theta);
void qe_trunk_conv_step(float *out, float *state, const float *x, const float *w, int C, int K);
void qe_trunk_l2norm(float *v, int n, float eps, float scale);
void qe_trunk_gates(float *g, float *beta, const float *a, const float *b, const float *A_log, const float *dt_bias,
                    int Hv);
void qe_trunk_recurrent_step(float *y, float *state, const float *q, const float *k, const float *v, const float *g,
                             const float *beta, int Hk, int Hv, int Dk, int Dv);

#ifdef __cplusplus
}
#endif
#endif
