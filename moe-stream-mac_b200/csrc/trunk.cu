/* trunk.cu: the whole model's trunk on the GPU (embedding row, RMSNorms, Gated DeltaNet and gated full-attention
 * layers, residuals, final norm, LM head), around the GPU MoE blocks, for one token per step.
 *
 * The contracts are the reference's (engine/include/ops.h, gdn.h, gdn_layer.h, attn_layer.h; engine/src/ops.c:5-14
 * RMSNorm, ops.c:75-93 RoPE, gdn.c conv step / L2 norm / gates / delta-rule recurrence, attn_layer.c gated GQA with
 * partial RoPE and an fp32 KV cache; model.c:135-157 the layer and model steps), as the host trunk of engine.cu
 * implements them. Element-wise arithmetic keeps the host trunk's fp32 operation order (separate multiplies and
 * adds, sequential sums where the host sums sequentially); norms and the attention softmax sum in double, with a
 * fixed tree order in place of the host's left-to-right order. The quantized projections and the LM head run on
 * the decode path's coalesced GEMV (qe_launch_dg_matvec; the general qe_launch_qmatvec for other shapes), with
 * qmat.c:36-46 semantics. Everything of a token stays on the device, and after the first step the whole step is
 * replayed from a CUDA graph; the logits are the only copy back.
 */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "qe_common.cuh"
#include "qe_kernels.h"
#include "trunk.h"

namespace {

constexpr int kNormThreads = 1024;

__device__ __forceinline__ float tk_silu(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float tk_sigmoid(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }

/* Block-wide sum of one double per thread, a fixed tree (shared memory red[blockDim.x / 32]). */
__device__ double tk_block_sum(double v, double *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(QE_FULL, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw; i++) t += red[i];
        red[0] = t;
    }
    __syncthreads();
    const double r = red[0];
    __syncthreads();
    return r;
}

/* Warp-wide sum of one double per lane (a fixed tree); every lane gets the result. */
__device__ __forceinline__ double tk_warp_sum(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(QE_FULL, v, o);
    return v;
}
__device__ __forceinline__ float tk_warp_sumf(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(QE_FULL, v, o));
    return v;
}

/* Code j of a row of a quantized matrix (LSB first within each 32-bit word, qgroup.c). */
__device__ __forceinline__ uint32_t tk_code(const uint32_t *row, int j, int bits) {
    return bits == 4 ? (row[j >> 3] >> ((j & 7) * 4)) & 15u : (row[j >> 2] >> ((j & 3) * 8)) & 255u;
}

/* Embedding row `token` dequantized (qmat_row.c): x[c] = q * scale + bias, MLX layout [rows][groups]. */
__global__ void tk_embed_kernel(QeQDev e, const int *__restrict__ tp, float *__restrict__ x) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= e.cols) return;
    const int token = tp[0];
    const int ng = e.cols / e.group_size, wpr = e.cols * e.bits / 32;
    const uint32_t *row = e.w + (size_t)token * wpr;
    const size_t g = (size_t)token * ng + c / e.group_size;
    x[c] = __fadd_rn(__fmul_rn((float)tk_code(row, c, e.bits), qe_bf16_to_f32(e.scales[g])), qe_bf16_to_f32(e.biases[g]));
}

/* RMSNorm of n values (ops.c:5-14): h = x (+ add, written to hout when add is given); out = h / sqrt(mean(h^2) +
 * eps) * w, the square sum in double. One CTA. */
__global__ void __launch_bounds__(kNormThreads) tk_rmsnorm_kernel(float *__restrict__ out, const float *x,
                                                                  const float *add, float *hout,
                                                                  const float *__restrict__ w, int n, float eps) {
    __shared__ double red[kNormThreads / 32];
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float h = add ? __fadd_rn(x[i], add[i]) : x[i];
        ss += (double)h * (double)h;
    }
    const double tot = tk_block_sum(ss, red);
    const float r = (float)sqrt(tot / n + (double)eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float h = add ? __fadd_rn(x[i], add[i]) : x[i];
        if (add) hout[i] = h;
        out[i] = __fmul_rn(__fdiv_rn(h, r), w[i]);
    }
}

/* ---------------------------------------------------------------- Gated DeltaNet (gdn.c, gdn_layer.c) */

/* Causal depthwise conv step over C channels (kernel K) and SiLU; the window of the last K-1 inputs moves by one.
 * One thread per channel (each owns its column of the state). */
__global__ void tk_conv_kernel(float *__restrict__ out, float *__restrict__ state, const float *__restrict__ x,
                               const float *__restrict__ w, int C, int K) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float acc = 0.0f;
    for (int j = 0; j + 1 < K; j++) acc = __fadd_rn(acc, __fmul_rn(state[(size_t)j * C + c], w[(size_t)c * K + j]));
    acc = __fadd_rn(acc, __fmul_rn(w[(size_t)c * K + K - 1], x[c]));
    out[c] = tk_silu(acc);
    for (int j = 0; j + 2 < K; j++) state[(size_t)j * C + c] = state[(size_t)(j + 1) * C + c];
    state[(size_t)(K - 2) * C + c] = x[c];
}

/* Per-head L2 norms of q (scaled by 1/sqrt(Dk)) and k, the gates g = exp(-exp(A_log) softplus(a + dt_bias)) and
 * beta = sigmoid(b) (gdn.c). Blocks 0..Hk-1: q heads, Hk..2Hk-1: k heads, block 2Hk: the gates. One warp each. */
__global__ void tk_gdn_prep_kernel(float *__restrict__ qk, int Hk, int Dk, float *__restrict__ g,
                                   float *__restrict__ beta, const float *__restrict__ a, const float *__restrict__ b,
                                   const float *__restrict__ A_log, const float *__restrict__ dt_bias, int Hv) {
    const int blk = blockIdx.x, lane = threadIdx.x;
    if (blk < 2 * Hk) {
        float *v = qk + (size_t)blk * Dk;   /* q heads first, then k heads (they are adjacent in the conv output) */
        double ss = 0.0;
        for (int i = lane; i < Dk; i += 32) ss += (double)v[i] * (double)v[i];
        ss = tk_warp_sum(ss);
        const double scale = blk < Hk ? (double)(1.0f / sqrtf((float)Dk)) : 1.0;   /* the host's float scale */
        const float f = (float)(scale / sqrt(ss + 1e-6));
        for (int i = lane; i < Dk; i += 32) v[i] = __fmul_rn(v[i], f);
    } else {
        for (int h = lane; h < Hv; h += 32) {
            const float t = __fadd_rn(a[h], dt_bias[h]);
            const float sp = t > 20.0f ? t : logf(__fadd_rn(1.0f, expf(t)));
            g[h] = expf(__fmul_rn(-expf(A_log[h]), sp));
            beta[h] = tk_sigmoid(b[h]);
        }
    }
}

/* The delta-rule step (gdn.c): per value head h and value row i (one warp, lanes over the key dimension):
 * S = g S; kv = S k; d = beta (v - kv); S += k d; y = S q. State [Hv][Dv][Dk]. */
__global__ void tk_recurrent_kernel(float *__restrict__ y, float *__restrict__ state, const float *__restrict__ q,
                                    const float *__restrict__ k, const float *__restrict__ v,
                                    const float *__restrict__ g, const float *__restrict__ beta, int Hk, int Hv,
                                    int Dk, int Dv) {
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (wid >= Hv * Dv) return;
    const int h = wid / Dv, i = wid % Dv, kh = h / (Hv / Hk);
    const float *kk = k + (size_t)kh * Dk, *kq = q + (size_t)kh * Dk;
    float *S = state + ((size_t)h * Dv + i) * Dk;
    const float gh = g[h];
    float kv = 0.0f;
    for (int j = lane; j < Dk; j += 32) {
        const float s = __fmul_rn(S[j], gh);
        S[j] = s;
        kv = __fadd_rn(kv, __fmul_rn(s, kk[j]));
    }
    kv = tk_warp_sumf(kv);
    const float d = __fmul_rn(__fsub_rn(v[(size_t)h * Dv + i], kv), beta[h]);
    float o = 0.0f;
    for (int j = lane; j < Dk; j += 32) {
        const float s = __fadd_rn(S[j], __fmul_rn(kk[j], d));
        S[j] = s;
        o = __fadd_rn(o, __fmul_rn(s, kq[j]));
    }
    o = tk_warp_sumf(o);
    if (lane == 0) y[(size_t)h * Dv + i] = o;
}

/* Gated RMSNorm per value head (gdn_layer.c): y_h = rmsnorm(y_h, norm_w) * silu(z_h). One warp per head. */
__global__ void tk_gated_norm_kernel(float *__restrict__ y, const float *__restrict__ z, const float *__restrict__ w,
                                     int Dv, float eps) {
    const int h = blockIdx.x, lane = threadIdx.x;
    float *yh = y + (size_t)h * Dv;
    const float *zh = z + (size_t)h * Dv;
    double ss = 0.0;
    for (int i = lane; i < Dv; i += 32) ss += (double)yh[i] * (double)yh[i];
    ss = tk_warp_sum(ss);
    const float r = (float)sqrt(ss / Dv + (double)eps);
    __syncwarp();
    for (int i = lane; i < Dv; i += 32) yh[i] = __fmul_rn(tk_silu(zh[i]), __fmul_rn(__fdiv_rn(yh[i], r), w[i]));
}

/* ---------------------------------------------------------------- gated full attention (attn_layer.c) */

/* RoPE on the first rot dims of one head (ops.c:75-93, rotate-half): angle pos * theta^(-2i/rot) in double. */
__device__ __forceinline__ void tk_rope_head(float *v, int rot, int pos, float theta, int lane) {
    const int half = rot / 2;
    for (int i = lane; i < half; i += 32) {
        const double ang = (double)pos * pow((double)theta, -2.0 * i / rot);
        const float cs = (float)cos(ang), sn = (float)sin(ang);
        const float a = v[i], b = v[i + half];
        v[i] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
        v[i + half] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
    }
}

/* Per-head RMSNorm of q (from the gated projection, stride 2D) and k, RoPE, and the KV-cache rows of position
 * pos = tp[1] (the step's token id and position live in device memory, so a captured step replays at any position). Blocks 0..Hq-1: q heads; Hq..Hq+Hkv-1: k heads (with their v rows). One warp each. */
__global__ void tk_attn_prep_kernel(float *__restrict__ q, const float *__restrict__ qg, float *__restrict__ kc,
                                    float *__restrict__ vc, const float *__restrict__ kx, const float *__restrict__ vx,
                                    const float *__restrict__ q_norm, const float *__restrict__ k_norm, int Hq,
                                    int Hkv, int D, int rot, const int *__restrict__ tp, float theta, float eps) {
    const int blk = blockIdx.x, lane = threadIdx.x, pos = tp[1];
    const bool isq = blk < Hq;
    const int h = isq ? blk : blk - Hq;
    const float *src = isq ? qg + (size_t)h * 2 * D : kx + (size_t)h * D;
    float *dst = isq ? q + (size_t)h * D : kc + ((size_t)pos * Hkv + h) * D;
    const float *w = isq ? q_norm : k_norm;
    double ss = 0.0;
    for (int i = lane; i < D; i += 32) ss += (double)src[i] * (double)src[i];
    ss = tk_warp_sum(ss);
    const float r = (float)sqrt(ss / D + (double)eps);
    for (int i = lane; i < D; i += 32) dst[i] = __fmul_rn(__fdiv_rn(src[i], r), w[i]);
    __syncwarp();
    tk_rope_head(dst, rot, pos, theta, lane);
    if (!isq)
        for (int i = lane; i < D; i += 32) vc[((size_t)pos * Hkv + h) * D + i] = vx[(size_t)h * D + i];
}

/* Causal attention of one query position over positions 0..n-1 (n = the position in tp[1], plus one) for head h (one CTA per head): scores q.k_t / sqrt(D)
 * (each a sequential sum over D), softmax with the max subtracted and exp and sum in double, o_i = sum_t p_t v_t,i
 * (sequential in t), times sigmoid(gate_i). sc: [Hq][max_len] scratch. */
__global__ void __launch_bounds__(kNormThreads) tk_attn_kernel(float *__restrict__ att, float *__restrict__ sc,
                                                               const float *__restrict__ q, const float *__restrict__ qg,
                                                               const float *__restrict__ kc,
                                                               const float *__restrict__ vc, int Hq, int Hkv, int D,
                                                               const int *__restrict__ tp, int max_len) {
    const int n = tp[1] + 1;
    __shared__ double red[kNormThreads / 32];
    __shared__ float mx_s;
    const int h = blockIdx.x, kvh = h / (Hq / Hkv);
    const float *qh = q + (size_t)h * D;
    float *s = sc + (size_t)h * max_len;
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    float mx = -INFINITY;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const float *kt = kc + ((size_t)t * Hkv + kvh) * D;
        float d = 0.0f;
        for (int i = 0; i < D; i++) d = __fadd_rn(d, __fmul_rn(qh[i], kt[i]));
        s[t] = __fmul_rn(d, inv_sqrt_d);
        mx = fmaxf(mx, s[t]);
    }
    /* block max */
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(QE_FULL, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = (double)mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -INFINITY;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, (float)red[i]);
        mx_s = m;
    }
    __syncthreads();
    const double m = (double)mx_s;
    double part = 0.0;
    for (int t = threadIdx.x; t < n; t += blockDim.x) part += exp((double)s[t] - m);
    const double sum = tk_block_sum(part, red);
    for (int t = threadIdx.x; t < n; t += blockDim.x) s[t] = (float)(exp((double)s[t] - m) / sum);
    __syncthreads();
    const float *gate = qg + (size_t)h * 2 * D + D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float o = 0.0f;
        for (int t = 0; t < n; t++) o = __fadd_rn(o, __fmul_rn(s[t], vc[((size_t)t * Hkv + kvh) * D + i]));
        att[(size_t)h * D + i] = __fmul_rn(o, tk_sigmoid(gate[i]));
    }
}

}  // namespace

/* ---------------------------------------------------------------- the device trunk */

struct TkLayerDev {
    bool linear = false;
    float *in_norm = nullptr, *post_norm = nullptr;
    QeQDev qkv{}, z{}, a{}, b{}, out{};
    float *conv_w = nullptr, *A_log = nullptr, *dt_bias = nullptr, *norm_w = nullptr;
    float *conv_state = nullptr, *rec_state = nullptr;
    QeQDev q{}, k{}, v{}, o{};
    float *q_norm = nullptr, *k_norm = nullptr;
    float *kc = nullptr, *vc = nullptr;                  /* [max_len][Hkv * D] */
    QeMoe *moe = nullptr;
};

struct GpuTrunk {
    TkDims d{};
    int dev = 0;
    cudaStream_t s = nullptr;
    std::vector<void *> allocs;
    QeQDev embed{}, lm_head{};
    float *final_norm = nullptr;
    std::vector<TkLayerDev> layers;
    float *x = nullptr, *h = nullptr, *t1 = nullptr, *t2 = nullptr;
    float *s1 = nullptr, *s2 = nullptr, *s3 = nullptr, *s4 = nullptr, *s5 = nullptr, *sc = nullptr;
    float *logits = nullptr;
    int *tp = nullptr;                 /* device: the step's token id and position */
    void *moe_ws = nullptr;            /* the MoE blocks' workspace (private: a captured step keeps its pointers) */
    int *tp_host = nullptr;            /* pinned host staging of tp */
    cudaGraphExec_t graph = nullptr;   /* the captured step (after the first eager step) */
    bool use_graph = true;
    ~GpuTrunk() {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(dev);
        if (s) cudaStreamSynchronize(s);
        if (graph) cudaGraphExecDestroy(graph);
        if (tp_host) cudaFreeHost(tp_host);
        for (void *p : allocs) cudaFree(p);
        if (s) cudaStreamDestroy(s);
        cudaSetDevice(cur);
    }
    template <typename T>
    T *alloc(size_t n) {
        void *p = nullptr;
        if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
        allocs.push_back(p);
        return static_cast<T *>(p);
    }
    float *upload(const float *src, size_t n) {
        float *p = alloc<float>(n);
        if (p && cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
        return p;
    }
    float *zeros(size_t n) {
        float *p = alloc<float>(n);
        if (p && cudaMemset(p, 0, n * sizeof(float)) != cudaSuccess) return nullptr;
        return p;
    }
    /* an MLX matrix to the device, same layout (scales [rows][groups]) */
    bool upload_q(const TkHostQ &h, QeQDev &q) {
        const size_t wb = (size_t)h.rows * ((size_t)h.cols * h.bits / 32) * 4, gb = (size_t)h.rows * (h.cols / h.gs) * 2;
        uint32_t *w = alloc<uint32_t>(wb / 4);
        uint16_t *sc = alloc<uint16_t>(gb / 2), *bi = alloc<uint16_t>(gb / 2);
        if (!w || !sc || !bi || cudaMemcpy(w, h.w, wb, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(sc, h.s, gb, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(bi, h.b, gb, cudaMemcpyHostToDevice) != cudaSuccess)
            return false;
        q.w = w; q.scales = sc; q.biases = bi;
        q.rows = h.rows; q.cols = h.cols; q.bits = h.bits; q.group_size = h.gs; q.scale_t = 0;
        return true;
    }
};

namespace {

/* y = W x on the device (one token) */
int tk_matvec(GpuTrunk *t, const QeQDev &m, const float *x, float *y) {
    const int rc = qe_launch_dg_matvec(&m, x, y, t->s);   /* the coalesced GEMV, or the general kernel */
    return rc == 1 ? qe_launch_qmatvec(&m, x, 1, y, t->s) : rc;
}

int tk_norm(GpuTrunk *t, float *out, const float *x, const float *add, float *hout, const float *w, int n) {
    tk_rmsnorm_kernel<<<1, kNormThreads, 0, t->s>>>(out, x, add, hout, w, n, t->d.eps);
    QE_CHECK(cudaGetLastError());
    return 0;
}

/* Gated DeltaNet layer on t1 -> t2 (gdn_layer.c; the host trunk's gdn_forward in engine.cu) */
int tk_gdn(GpuTrunk *t, TkLayerDev &L) {
    const TkDims &d = t->d;
    const int KD = d.lin_Hk * d.lin_Dk, VD = d.lin_Hv * d.lin_Dv, C = 2 * KD + VD;
    float *qkv = t->s1, *cv = t->s2, *z = t->s3, *y = t->s4, *a = t->s5, *b = t->s5 + d.lin_Hv,
          *g = t->s5 + 2 * d.lin_Hv, *beta = t->s5 + 3 * d.lin_Hv;
    if (tk_matvec(t, L.qkv, t->t1, qkv) || tk_matvec(t, L.z, t->t1, z) || tk_matvec(t, L.a, t->t1, a) ||
        tk_matvec(t, L.b, t->t1, b))
        return -1;
    tk_conv_kernel<<<(C + 127) / 128, 128, 0, t->s>>>(cv, L.conv_state, qkv, L.conv_w, C, d.conv_K);
    tk_gdn_prep_kernel<<<2 * d.lin_Hk + 1, 32, 0, t->s>>>(cv, d.lin_Hk, d.lin_Dk, g, beta, a, b, L.A_log, L.dt_bias,
                                                          d.lin_Hv);
    const int warps = d.lin_Hv * d.lin_Dv;
    tk_recurrent_kernel<<<(warps + 7) / 8, 256, 0, t->s>>>(y, L.rec_state, cv, cv + KD, cv + 2 * KD, g, beta, d.lin_Hk,
                                                           d.lin_Hv, d.lin_Dk, d.lin_Dv);
    tk_gated_norm_kernel<<<d.lin_Hv, 32, 0, t->s>>>(y, z, L.norm_w, d.lin_Dv, d.eps);
    QE_CHECK(cudaGetLastError());
    return tk_matvec(t, L.out, y, t->t2);
}

/* Gated full attention on t1 -> t2 at the step's position (attn_layer.c; the host trunk's attn_forward) */
int tk_attn(GpuTrunk *t, TkLayerDev &L) {
    const TkDims &d = t->d;
    float *qg = t->s1, *q = t->s2, *att = t->s3, *kx = t->s4, *vx = t->s5;
    if (tk_matvec(t, L.q, t->t1, qg) || tk_matvec(t, L.k, t->t1, kx) || tk_matvec(t, L.v, t->t1, vx)) return -1;
    tk_attn_prep_kernel<<<d.Hq + d.Hkv, 32, 0, t->s>>>(q, qg, L.kc, L.vc, kx, vx, L.q_norm, L.k_norm, d.Hq, d.Hkv, d.D,
                                                       d.rot, t->tp, d.theta, d.eps);
    tk_attn_kernel<<<d.Hq, kNormThreads, 0, t->s>>>(att, t->sc, q, qg, L.kc, L.vc, d.Hq, d.Hkv, d.D, t->tp, d.max_len);
    QE_CHECK(cudaGetLastError());
    return tk_matvec(t, L.o, att, t->t2);
}

}  // namespace

GpuTrunk *qe_gtrunk_create(const TkDims &d, const TkHostQ &embed, const TkHostQ &lm_head, const float *final_norm,
                           const std::vector<TkLayerHost> &layers, int dev) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cudaSetDevice(dev) != cudaSuccess) {
        fprintf(stderr, "qengine_b200: GPU trunk: device %d unavailable\n", dev);
        return nullptr;
    }
    GpuTrunk *t = new GpuTrunk();
    t->d = d;
    t->dev = dev;
    bool ok = cudaStreamCreateWithFlags(&t->s, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && t->upload_q(embed, t->embed) && t->upload_q(lm_head, t->lm_head) &&
         (t->final_norm = t->upload(final_norm, (size_t)d.hidden)) != nullptr;
    const int KD = d.lin_Hk * d.lin_Dk, VD = d.lin_Hv * d.lin_Dv, C = 2 * KD + VD;
    const size_t QD = (size_t)d.Hq * d.D, KVD = (size_t)d.Hkv * d.D;
    for (const TkLayerHost &h : layers) {
        if (!ok) break;
        TkLayerDev L;
        L.linear = h.linear;
        L.moe = h.moe;
        ok = (L.in_norm = t->upload(h.in_norm, (size_t)d.hidden)) && (L.post_norm = t->upload(h.post_norm, (size_t)d.hidden));
        if (ok && h.linear) {
            ok = t->upload_q(h.qkv, L.qkv) && t->upload_q(h.z, L.z) && t->upload_q(h.a, L.a) && t->upload_q(h.b, L.b) &&
                 t->upload_q(h.out, L.out) && (L.conv_w = t->upload(h.conv_w, (size_t)C * d.conv_K)) &&
                 (L.A_log = t->upload(h.A_log, (size_t)d.lin_Hv)) && (L.dt_bias = t->upload(h.dt_bias, (size_t)d.lin_Hv)) &&
                 (L.norm_w = t->upload(h.norm_w, (size_t)d.lin_Dv)) &&
                 (L.conv_state = t->zeros((size_t)(d.conv_K - 1) * C)) &&
                 (L.rec_state = t->zeros((size_t)d.lin_Hv * d.lin_Dv * d.lin_Dk));
        } else if (ok) {
            ok = t->upload_q(h.q, L.q) && t->upload_q(h.k, L.k) && t->upload_q(h.v, L.v) && t->upload_q(h.o, L.o) &&
                 (L.q_norm = t->upload(h.q_norm, (size_t)d.D)) && (L.k_norm = t->upload(h.k_norm, (size_t)d.D)) &&
                 (L.kc = t->zeros((size_t)d.max_len * KVD)) && (L.vc = t->zeros((size_t)d.max_len * KVD));
        }
        t->layers.push_back(L);
    }
    const size_t H = (size_t)d.hidden;
    const size_t big = std::max(std::max((size_t)C, 2 * QD), std::max(H, (size_t)VD));
    ok = ok && (t->x = t->zeros(H)) && (t->h = t->zeros(H)) && (t->t1 = t->zeros(H)) && (t->t2 = t->zeros(H)) &&
         (t->s1 = t->zeros(big)) && (t->s2 = t->zeros(big)) && (t->s3 = t->zeros(big)) &&
         (t->s4 = t->zeros(std::max(big, KVD))) && (t->s5 = t->zeros(std::max((size_t)4 * d.lin_Hv, KVD))) &&
         (t->sc = t->zeros((size_t)d.Hq * d.max_len)) && (t->logits = t->zeros((size_t)d.vocab)) &&
         (t->tp = t->alloc<int>(2)) != nullptr && cudaMallocHost((void **)&t->tp_host, 2 * sizeof(int)) == cudaSuccess;
    size_t wsb = 0;
    for (const TkLayerHost &h : layers) wsb = std::max(wsb, qe_moe_ws_bytes(h.moe, 1));
    ok = ok && wsb > 0 && (t->moe_ws = t->alloc<char>(wsb)) != nullptr;
    const char *ge = getenv("QE_TRUNK_GRAPH");   /* 0: launch the step's kernels one by one */
    t->use_graph = !(ge && !strcmp(ge, "0"));
    cudaSetDevice(cur);
    if (!ok) {
        fprintf(stderr, "qengine_b200: GPU trunk: upload failed (%s)\n", cudaGetErrorString(cudaGetLastError()));
        delete t;
        return nullptr;
    }
    return t;
}

namespace {

/* Enqueue one token's step on t->s (the token id and position already in t->tp); no host work that a graph replay
 * would skip, except the statistics note when `note` (eager steps). */
int tk_step(GpuTrunk *t, bool note) {
    const TkDims &d = t->d;
    const int H = d.hidden;
    int rc = 0;
    tk_embed_kernel<<<(H + 255) / 256, 256, 0, t->s>>>(t->embed, t->tp, t->x);
    /* per layer (model.c:135-146): x1 = x + mixer(norm(x)); x = x1 + moe(norm(x1)). The residual of the previous
     * layer's MoE block is added inside the next norm (t2 holds that block's output, h its input). */
    for (size_t l = 0; l < t->layers.size() && !rc; l++) {
        TkLayerDev &L = t->layers[l];
        rc = l == 0 ? tk_norm(t, t->t1, t->x, nullptr, nullptr, L.in_norm, H)
                    : tk_norm(t, t->t1, t->h, t->t2, t->x, L.in_norm, H);
        if (!rc) rc = L.linear ? tk_gdn(t, L) : tk_attn(t, L);
        if (!rc) rc = tk_norm(t, t->t1, t->x, t->t2, t->h, L.post_norm, H);
        if (!rc) rc = qe_moe_forward_device_ws(L.moe, 1, t->t1, t->t2, t->moe_ws, t->s);
        if (!rc && note) rc = qe_moe_note_device_forward(L.moe, 1, t->moe_ws, t->s);
    }
    /* the last block's residual, the final norm and the LM head (model.c:150-157) */
    if (!rc) rc = tk_norm(t, t->t1, t->h, t->t2, t->x, t->final_norm, H);
    if (!rc) rc = tk_matvec(t, t->lm_head, t->t1, t->logits);
    return rc;
}

/* Capture the step in a CUDA graph (after an eager step has sized every workspace). */
int tk_capture(GpuTrunk *t) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(t->s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -1;
    const int rc = tk_step(t, false);
    const cudaError_t e = cudaStreamEndCapture(t->s, &g);
    if (rc || e != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return -1;
    }
    const cudaError_t ie = cudaGraphInstantiate(&t->graph, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        t->graph = nullptr;
        cudaGetLastError();
        return -1;
    }
    return 0;
}

}  // namespace

int qe_gtrunk_forward(GpuTrunk *t, int token, int pos, float *logits) {
    const TkDims &d = t->d;
    if (token < 0 || token >= d.vocab || pos < 0 || pos >= d.max_len) return -1;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cudaSetDevice(t->dev) != cudaSuccess) return -1;
    t->tp_host[0] = token;
    t->tp_host[1] = pos;
    int rc = cudaMemcpyAsync(t->tp, t->tp_host, 2 * sizeof(int), cudaMemcpyHostToDevice, t->s) != cudaSuccess;
    /* QE_TRACE needs each layer's routing read back between the layers: eager steps then */
    const bool graph = t->use_graph && !getenv("QE_TRACE");
    if (!rc && graph && t->graph) {
        rc = cudaGraphLaunch(t->graph, t->s) != cudaSuccess;
        for (size_t l = 0; l < t->layers.size() && !rc; l++)
            rc = qe_moe_note_device_forward(t->layers[l].moe, 1, nullptr, nullptr);
    } else if (!rc) {
        rc = tk_step(t, true);
    }
    if (!rc && cudaMemcpyAsync(logits, t->logits, sizeof(float) * d.vocab, cudaMemcpyDeviceToHost, t->s) != cudaSuccess)
        rc = -1;
    if (cudaStreamSynchronize(t->s) != cudaSuccess) rc = -1;
    /* the first step ran eagerly (and sized the MoE workspaces): capture the step for the next ones */
    if (!rc && graph && !t->graph && tk_capture(t)) t->use_graph = false;
    cudaSetDevice(cur);
    return rc ? -1 : 0;
}

int qe_gtrunk_reset(GpuTrunk *t) {
    const TkDims &d = t->d;
    const int KD = d.lin_Hk * d.lin_Dk, VD = d.lin_Hv * d.lin_Dv, C = 2 * KD + VD;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(t->dev);
    int rc = 0;
    for (TkLayerDev &L : t->layers)
        if (L.linear)
            rc |= cudaMemsetAsync(L.conv_state, 0, sizeof(float) * (size_t)(d.conv_K - 1) * C, t->s) != cudaSuccess ||
                  cudaMemsetAsync(L.rec_state, 0, sizeof(float) * (size_t)d.lin_Hv * d.lin_Dv * d.lin_Dk, t->s) !=
                      cudaSuccess;
    rc |= cudaStreamSynchronize(t->s) != cudaSuccess;
    cudaSetDevice(cur);
    return rc ? -1 : 0;
}

void qe_gtrunk_free(GpuTrunk *t) { delete t; }
