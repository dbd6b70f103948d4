/* trunk.h: the GPU trunk of the whole-model API (trunk.cu), as engine.cu drives it. Internal to the library. */
#ifndef QE_TRUNK_H
#define QE_TRUNK_H
#include <stdint.h>

#include <vector>

#include "../../include/qe_moe.h"

/* One MLX affine quantized matrix in host memory (the checkpoint mapping): codes [rows][cols*bits/32] words,
 * bf16 scales and biases [rows][cols/group]. */
struct TkHostQ {
    const uint32_t *w = nullptr;
    const uint16_t *s = nullptr, *b = nullptr;
    int rows = 0, cols = 0, bits = 0, gs = 0;
};

struct TkDims {
    int hidden, vocab, Hq, Hkv, D, rot, lin_Hk, lin_Hv, lin_Dk, lin_Dv, conv_K, max_len;
    float eps, theta;
};

/* One layer's trunk tensors (host memory; copied to the device at create) and its MoE handle. */
struct TkLayerHost {
    bool linear = false;
    const float *in_norm = nullptr, *post_norm = nullptr;
    TkHostQ qkv, z, a, b, out;                               /* Gated DeltaNet */
    const float *conv_w = nullptr, *A_log = nullptr, *dt_bias = nullptr, *norm_w = nullptr;
    TkHostQ q, k, v, o;                                      /* gated attention */
    const float *q_norm = nullptr, *k_norm = nullptr;
    QeMoe *moe = nullptr;
};

/* After a device forward inside a caller's own step: read statistics and (with a stream) QE_TRACE records, as
 * qe_moe_forward keeps them; ws: the workspace the forward used, or null for the device's shared one. And the
 * device forward on a caller's workspace (qe_moe_ws_bytes(m, T) bytes), stable under graph capture (qe_moe.cu). */
extern "C" int qe_moe_note_device_forward(QeMoe *m, int T, void *ws, void *stream);
extern "C" size_t qe_moe_ws_bytes(const QeMoe *m, int T);
extern "C" int qe_moe_forward_device_ws(QeMoe *m, int T, const float *x, float *out, void *ws, void *stream);

struct GpuTrunk;
/* Upload the trunk to CUDA device `dev` (the MoE handles' device). NULL on failure (reason on stderr). */
GpuTrunk *qe_gtrunk_create(const TkDims &d, const TkHostQ &embed, const TkHostQ &lm_head, const float *final_norm,
                           const std::vector<TkLayerHost> &layers, int dev);
/* One token at position pos (0 <= pos < max_len, token < vocab): the logits to host memory. 0 ok, -1 error. */
int qe_gtrunk_forward(GpuTrunk *t, int token, int pos, float *logits);
/* Clear the recurrent and convolution states (the KV caches are only read below the position). */
int qe_gtrunk_reset(GpuTrunk *t);
void qe_gtrunk_free(GpuTrunk *t);

#endif
