/* qe_kernels.h: internal launchers shared by the .cu files of libqengine_b200 (not part of the C ABI). */
#ifndef QE_KERNELS_H
#define QE_KERNELS_H
#include <cuda_runtime.h>
#include <stdint.h>

/* One quantized matrix in the MLX affine layout (engine/include/qmat.h:3-11), resident in HBM.
 * For routed experts the pointers cover all E experts: expert e starts at w + e*rows*wpr words and at
 * scales/biases + e*rows*ngroups halves (engine/src/loader.c:35-41). */
struct QeQDev {
    const uint32_t *w;
    const uint16_t *scales;
    const uint16_t *biases;
    int rows, cols, bits, group_size;
    int scale_t;   /* 0: MLX layout [n][rows][groups]; 1: expert kernels' layout [n][groups][rows] */
};

/* Routing: fp32 router logits for E experts plus one extra column (index E) holding the shared-expert
 * gate logit, logits[T][E+1]. qe_launch_router_f32 returns the number of kernels it launched, or -1. */
int qe_launch_router_f32(const float *W /*[E+1][H]*/, const float *bias /*[E] or null*/, const float *x,
                         int T, int H, int E, float *logits,
                         float *part /* [ceil(H/64)][T][E+1] scratch for the chunk-split prefill GEMM, or null */,
                         const float *Wd /* [H][qe_router_wd_rows(E)][2] duplicated weights, or null */,
                         float *xt /* [H][T rounded up to 4] scratch for the transposed batch, or null */,
                         cudaStream_t s);
/* Rows and contents of the paired-FMA prefill router's weight copy Wd[k][row][2] (rows past E are zero; when
 * E + 1 = 64n + 1 the gate row E is read from W instead). */
int qe_router_wd_rows(int E);
int qe_launch_router_wd_fill(const float *W, int H, int E, float *Wd, cudaStream_t s);
int qe_launch_router_qmat(const QeQDev *router /*[E][H]*/, const QeQDev *sh_router /*[1][H]*/, const float *x,
                          int T, int H, int E, float *logits, cudaStream_t s);
int qe_launch_route_topk(const float *logits, int ld, int T, int E, int k, int32_t *idx, float *score,
                         float *probs /* [T][E] or null */, cudaStream_t s);

/* Bucketing: expert-sorted (token, slot) pairs and the work lists of the expert kernels. */
struct QeBuckets {
    int32_t *counts;      /* [E+1]                                            */
    int32_t *offsets;     /* [E+2]                                            */
    int32_t *cursor;      /* [E+1]                                            */
    int32_t *pairs;       /* [T*(k+1)] pair ids p = t*(k+1)+j, sorted by slot */
    int32_t *slot_expert; /* [E+1] active slots -> expert id (E = shared)     */
    int32_t *slot_items;  /* [2][E+2] per-slot work-item prefix, gate/up & down */
    int32_t *n_active;    /* [3]: active slots, gate/up items, down items     */
    int4 *chunks;         /* [T*(k+1)] or null: with one tile per expert, chunk c of the gate/up item list as
                             {expert, first bucket position, tokens} (the grouped GEMVs' work list) */
};
/* The shared expert's bucket holds rows [shared_first, shared_first + shared_tokens) of the batch. */
int qe_launch_bucket(const int32_t *idx, int T, int E, int k, int shared_tokens, int tiles_gu, int tiles_sh_gu,
                     int tiles_dn, int chunk, const QeBuckets *b, cudaStream_t s, int shared_first = 0);

/* Expert kernels (mma.sync split-bf16 path). */
struct QeExpertArgs {
    QeQDev gate, up, down;            /* routed experts, [E][...]           */
    QeQDev sh_gate, sh_up, sh_down;   /* shared expert                      */
    int E, k, hidden, inter, sh_inter;
};
int qe_launch_gateup(const QeExpertArgs *a, const float *x, const QeBuckets *b, int T, float *h3 /*[T*(k+1)][I]*/,
                     int ldh, int grid, cudaStream_t s);
int qe_launch_down(const QeExpertArgs *a, const float *h3, int ldh, const QeBuckets *b, int T,
                   float *ybuf /*[T*(k+1)][H]*/, int grid, cudaStream_t s);
int qe_launch_combine(const float *ybuf, const float *score, const float *logits, int ld_logits, int T, int E,
                      int k, int H, float *out, cudaStream_t s);
/* Expert-parallel variants: the routed slots whose idx is >= 0 (slot order), and/or the gated shared expert. */
int qe_launch_combine_sel(const float *ybuf, const int32_t *idx, const float *score, const float *logits,
                          int ld_logits, int T, int E, int k, int H, int with_routed, int with_shared, float *out,
                          cudaStream_t s);

int qe_launch_combine_sel_scatter(const float *ybuf, const int32_t *idx, const float *score, int T, int k, int H,
                                  float *const *dst_base /* device [G] */, int row0, int Tblk, int self,
                                  cudaStream_t s);

/* Decode GEMVs (decode.cu): gate/up + SwiGLU per (token, slot) pair into h3 [T*(k+1)][ldh], then down + the
 * weighted combine (top-k order, then the gated shared expert) into out [T][hidden]. */
bool qe_decode_supported(const QeExpertArgs *a);
int qe_launch_decode_fused(const QeExpertArgs *a, const float *W, const float *bias, const float *x, int T,
                           float *logits, int32_t *idx, float *score, float *h3, int ldh, float *out, unsigned *bar,
                           int sms, cudaStream_t s);
int qe_decode_error(void);
int qe_decode_error_reset(void);
int qe_launch_decode_gateup(const QeExpertArgs *a, const float *x, const int32_t *idx, int T, float *h3, int ldh,
                            cudaStream_t s);
int qe_launch_decode_down_combine(const QeExpertArgs *a, const float *h3, int ldh, const int32_t *idx,
                                  const float *score, const float *logits, int ld_logits, int T, float *out,
                                  cudaStream_t s);

/* Generic quantized matrix-vector products (engine/src/qmat.c:15-49 semantics) over T vectors. */
int qe_launch_qmatvec(const QeQDev *m, const float *x, int T, float *y, cudaStream_t s);
/* y = W x on the coalesced decode GEMV (decode.cu): 1 when the shape is not covered, 0 launched, -1 error. */
int qe_launch_dg_matvec(const QeQDev *m, const float *x, float *y, cudaStream_t s);

/* Synthetic weights generated in HBM (csrc/synth.h). */
int qe_launch_synth_qmat(uint64_t seed, uint32_t block, uint32_t stream, int first, int n, int rows, int cols,
                         int bits, int gs, int scale_t, uint32_t *w, uint16_t *sc, uint16_t *bi, cudaStream_t s);
/* [n][rows][groups] -> [n][groups][rows] for a bf16 scale or bias tensor */
int qe_launch_transpose_groups(const uint16_t *src, uint16_t *dst, int n, int rows, int groups, cudaStream_t s);
int qe_launch_synth_normal(uint64_t seed, uint32_t block, uint32_t stream, size_t n, float sigma_c, float *out,
                           cudaStream_t s);

int qe_num_sms(void);
/* Host threads for the library's CPU-side work (qe_set_threads; default: the hardware threads). */
int qe_host_thread_count(void);

/* Tensor-core (tcgen05) prefill path, expert_tc.cu. */
#include <cuda_fp16.h>
/* Split activations of the tensor-core path: per group of 64 inputs, v * 2^e = hi + lo (fp16). */
struct QeTcBufs {
    __half *act;            /* gate/up input [2][T][hidden] */
    float *actsum, *actinv; /* [T][hidden/64]: group sums of x, 2^-e */
    __half *h3s;            /* down input [2][npairs][ldh] */
    float *h3sum, *h3inv;   /* [npairs][ldh/64] */
    int ldh;
};
bool qe_tc_supported(const QeExpertArgs *a);
size_t qe_tc_map_bytes(void);
int qe_tc_weight_maps(const QeQDev *q, int n_experts, void *codes_map, void *sc_map, void *bi_map);
int qe_launch_tc_prep(const QeExpertArgs *a, const float *x, int T, const QeTcBufs *tb, cudaStream_t s);
int qe_launch_split_rows(int bits, const float *src, int K, int rows, __half *act, float *asum, float *ainv,
                         cudaStream_t s);
/* Expert-centric grouped GEMVs for batched decode (group_gemv.cu), on activations split as for the tcgen05
 * kernels. */
bool qe_group_supported(const QeExpertArgs *a);
int qe_group_tokens(void);   /* tokens per chunk of the bucket lists the grouped GEMVs read */
int qe_launch_group_gateup(const QeExpertArgs *a, const QeTcBufs *tb, int T, const QeBuckets *b, int sms, float *h3,
                           int ldh, cudaStream_t s);
int qe_launch_group_down(const QeExpertArgs *a, const QeTcBufs *tb, int npairs, const QeBuckets *b, int sms,
                         float *ybuf, cudaStream_t s);
int qe_launch_tc_gateup(const QeExpertArgs *a, const void *maps, const float *x, const QeBuckets *b, int T, int tn,
                        const QeTcBufs *t, int grid, cudaStream_t s);
int qe_launch_tc_down(const QeExpertArgs *a, const void *maps, const QeBuckets *b, int T, int tn, const QeTcBufs *t,
                      float *ybuf, int grid, cudaStream_t s);
int qe_tc_error(void);
int qe_tc_error_reset(void);
int qe_tc_bm(void);
int qe_tc_tokens_per_tile(int T, int top_k, int E);

#endif
