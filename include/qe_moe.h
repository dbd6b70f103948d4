/* qe_moe.h: C ABI of libqengine_b200, the B200 routed-MoE block (one qwen3_5_moe sparse MoE layer).
 *
 * Drop-in boundary. In hatim-mlf/moe-stream-mac the block is
 *     int moe_layer_step(float *out, const float *x, const MoeWeights *w, float *scratch);
 * (engine/include/moe_layer.h:33, implemented at engine/src/moe_layer.c:66-89), called once per token and
 * layer by model.c:layer_step (model.c:135-148) and, through the engine's C API (engine/include/qengine.h),
 * by engine/cli/qchat.py via ctypes. This header is the same operation as a handle-based library in the
 * conventions of that C API: opaque handle, NULL on a failed load with the reason on stderr, int return
 * codes 0 = ok / -1 = error with outputs untouched, caller-owned input/output buffers, library-owned
 * weights. The experts stay resident in HBM (the reference preads the 8 selected experts from SSD per
 * token, engine/src/expert_store.c:54-61). There is no CPU fallback: without a usable GPU, create returns
 * NULL.
 *
 * Threading: a handle is not thread-safe. All handles on one device share one scratch workspace and one
 * stream for the host-buffer calls, so calls must not overlap (the reference is single-caller too).
 */
#ifndef QE_MOE_H
#define QE_MOE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct QeMoe QeMoe;

enum { QE_ROUTER_F32 = 0, QE_ROUTER_QMAT = 1 };

/* Block shape: the MoeWeights fields of engine/include/moe_layer.h:19-20 plus the experts' affine
 * quantization (bits 4 or 8, group_size 32/64/128: engine/src/qmat.c:16-20) and the router kind. */
typedef struct {
    int hidden, E, top_k, inter, sh_inter;
    int bits, group_size;
    int router_mode;      /* QE_ROUTER_F32: fp32 router [E][hidden] + fp32 shared gate [hidden];
                             QE_ROUTER_QMAT: quantized router QMat [E][hidden] + shared gate QMat [1][hidden]
                             (the checkpoint layout, moe_layer.h:13 and :18) */
    int router_bits;      /* bits of the quantized router (QE_ROUTER_QMAT) */
    int max_tokens;       /* tokens per internal pass (scratch sizing); forward accepts any T >= 1 */
    int device;           /* CUDA device ordinal */
    int layer;            /* layer id written to the QE_TRACE routing trace (moe_layer.c:57-64) */
    int ep_rank, ep_size; /* expert parallelism: this handle holds routed experts [ep_rank*E/ep_size,
                             (ep_rank+1)*E/ep_size) plus the router and the shared expert (replicated).
                             ep_size 0 or 1 = all experts (then ep_rank must be 0). ep_size must divide E
                             unless a placement is given. */
    const int32_t *placement; /* NULL: the contiguous ranges above. Else a host table [ep_size][slots], the
                             same on every rank: row r lists the global expert ids rank r holds (-1 = empty
                             slot; no id twice in a row; every id in at least one row). An expert held by
                             n > 1 ranks (a replicated hot expert) serves each token on one of them, chosen
                             by the rule under QE_EP_ROUTED below. Needs ep_size > 1. Copied at create. */
    int slots;            /* columns of placement */
} QeMoeConfig;

/* Expert placement: a (token, expert) assignment goes to rank reps[e][(t + src) % nrep[e]], where reps[e]
 * lists the nrep[e] ranks holding e in ascending order, t is the token's row on its source rank and src is
 * that rank (0 in the replicated step, where every rank holds the same rows). In the slot lists that
 * qe_moe_ep_pack_device / qe_moe_ep_dispatch_p2p write for destination d, the ids of the slots routed to d
 * carry QE_EP_ROUTED and the other slots are -1. */
#define QE_EP_ROUTED 0x40000000

/* One quantized tensor in the MLX affine layout (engine/include/qmat.h:3-11): uint32 codes
 * [n][rows][cols*bits/32] (LSB first), bf16 scales and biases [n][rows][cols/group_size]. */
typedef struct {
    const uint32_t *w;
    const uint16_t *scales;
    const uint16_t *biases;
} QeQTensor;

/* Host pointers to one block's weights (MoeWeights, moe_layer.h:12-21; names of model.c:52-64). */
typedef struct {
    const float *router_f32;   /* [E][hidden]                      (QE_ROUTER_F32)  */
    const float *router_bias;  /* [E] added to the fp32 logits, or NULL                */
    const float *sh_gate_f32;  /* [hidden]                          (QE_ROUTER_F32)  */
    QeQTensor router_q;        /* mlp.gate            [E][hidden]  (QE_ROUTER_QMAT) */
    QeQTensor sh_router_q;     /* mlp.shared_expert_gate [1][hidden] (QE_ROUTER_QMAT) */
    QeQTensor gate, up, down;  /* mlp.switch_mlp.{gate,up,down}_proj [E][...]          */
    QeQTensor sh_gate, sh_up, sh_down; /* mlp.shared_expert.{gate,up,down}_proj        */
} QeMoeWeights;

/* Validate cfg, copy the weights into HBM. NULL on failure (stderr says why). Replaces load_moe
 * (engine/src/model.c:52-82) + expert_tensor_open (engine/src/expert_store.c:21-36). */
QeMoe *qe_moe_create(const QeMoeConfig *cfg, const QeMoeWeights *w);

/* Same block generated directly in HBM from the seeded generator of csrc/synth.h (bit-identical to the
 * CPU checker's copy). router_bias: [E] host array or NULL. */
QeMoe *qe_moe_create_synthetic(const QeMoeConfig *cfg, uint64_t seed, uint32_t block, const float *router_bias);

/* The block of one layer from an MLX checkpoint directory (every *.safetensors shard in `dir`), as the
 * reference's load_moe reads it (engine/src/model.c:52-70, engine/src/loader.c:16-41,
 * engine/src/io/k3_st.c:509): tensors <prefix>.switch_mlp.{gate,up,down}_proj, <prefix>.gate,
 * <prefix>.shared_expert.{gate,up,down}_proj, <prefix>.shared_expert_gate, each .weight/.scales/.biases.
 * prefix is e.g. "language_model.model.layers.3.mlp". From cfg only top_k, group_size, max_tokens, device,
 * layer and ep_rank/ep_size are taken; hidden, E, inter, sh_inter, bits and the quantized router's bits come
 * from the tensor shapes (a nonzero cfg value that disagrees is refused). NULL on failure (stderr says why). */
QeMoe *qe_moe_open_safetensors(const char *dir, const char *prefix, const QeMoeConfig *cfg);

/* dtype (e.g. "U32", NUL-terminated, <= 7 chars) and shape[ndim] (ndim <= 8) of one tensor of a checkpoint
 * directory; host only, no GPU needed. 0 ok, -1 if missing or malformed. */
int qe_safetensors_tensor_info(const char *dir, const char *name, char *dtype, int64_t *shape, int *ndim);

void qe_moe_free(QeMoe *m);

/* out[T][hidden] = moe(x[T][hidden]) for T >= 1 independent tokens, host buffers (x, out may not alias).
 * Replaces T calls of moe_layer_step (engine/src/moe_layer.c:66-89). 0 ok, -1 error (out untouched).
 * A handle holding a subset of the experts (ep_size > 1) refuses it: use the qe_moe_ep_* calls. */
int qe_moe_forward(QeMoe *m, int T, const float *x, float *out);
/* Pipelined qe_moe_forward: enqueues the copy of x[T][hidden] to the device, the forward and the copy of
 * out[T][hidden] back, and returns without waiting; qe_moe_forward_wait(m) waits for every such call on m's
 * device. Consecutive calls overlap their copies with each other's kernels (two staging slots per device; x
 * and out in pinned host memory for the copies to be asynchronous). x and out must stay valid and out unread
 * until the wait. The forward is replayed from CUDA graphs that the handle's first call with a given T
 * captures for both staging slots at once (that call synchronises the device; so does a call that grows the
 * staging buffers); every later call with that T only enqueues work. Same results as qe_moe_forward;
 * T <= max_tokens; the read statistics are not updated and the routing trace (QE_TRACE) is not written.
 * No reference counterpart (moe_layer_step returns with out written). 0 ok, -1 error. */
int qe_moe_forward_async(QeMoe *m, int T, const float *x, float *out);
int qe_moe_forward_wait(QeMoe *m);

/* Same on device buffers of m's device, enqueued on `stream` (a cudaStream_t, NULL = legacy default),
 * no host synchronisation. */
int qe_moe_forward_device(QeMoe *m, int T, const float *x, float *out, void *stream);

/* qe_moe_forward_device of T tokens on fixed device buffers x/out, captured once into a CUDA graph and replayed
 * by qe_moe_graph_launch on any stream of the handle's device (decode loops: the same T every step, no host
 * launch overhead per kernel). The graph has its own scratch; the handle must outlive it, and replays of one
 * graph must not overlap. No reference counterpart. NULL / -1 on failure. */
typedef struct QeMoeGraph QeMoeGraph;
QeMoeGraph *qe_moe_graph_create(QeMoe *m, int T, const float *x, float *out);
int qe_moe_graph_launch(QeMoeGraph *g, void *stream);
void qe_moe_graph_free(QeMoeGraph *g);

/* Routing only (moe_layer.c:29-37): idx[T][top_k] expert ids, score[T][top_k] renormalised weights,
 * host buffers. */
int qe_moe_route(QeMoe *m, int T, const float *x, int32_t *idx, float *score);

/* ---- expert parallelism (one process and one handle per GPU; the caller runs the collectives) ----
 * No counterpart in the reference (single-process, engine/src/moe_layer.c). Experts are sharded by id:
 * expert e lives on rank e / (E/ep_size), or where cfg.placement puts it. All buffers are device buffers on
 * the handle's device, enqueued on `stream` (a cudaStream_t). A token's slot list "meta" is int32 [2*top_k]:
 * the k global expert ids (-1 = empty slot) followed by the k renormalised scores' float bits.
 *
 * Token-sharded step (prefill batches, C4/C5 style), per rank with its own T tokens, G = ep_size:
 *   qe_moe_ep_route_device    route x, write meta[T][2k], and the gated shared-expert term shared[T][h]
 *   qe_moe_ep_pack_device     send_x[G][T][h], send_meta[G][T][2k]: rows of the tokens with >= 1 slot routed
 *                             to rank d go to block d in token order (ids of the slots routed elsewhere -1,
 *                             the others tagged QE_EP_ROUTED), the rest of the block is padding (meta ids
 *                             -1); home[G][T] = a token's row in block d or -1; counts[G] rows per block
 *   (caller) all_to_all of send_x and send_meta in equal blocks of T rows
 *   qe_moe_ep_experts_device  partial[n][h] for received rows: sum over the slots routed to this rank, in
 *                             slot order, of score * expert(x)  (rows without such slots give 0); untagged
 *                             ids (the replicated step's own meta) count where their replica is this rank
 *   (caller) all_to_all of partial back to the home ranks
 *   qe_moe_ep_combine_device  out[t] = (sum over d ascending of part[d][home[d][t]]) + shared[t]
 * Replicated step (decode: every rank holds the same T tokens): route, experts on the own meta, an all-gather
 * of the partials into part[G][T][h], combine with home = NULL (part[d][t]).
 * With ep_size = 1 the token-sharded step gives results bit-identical to qe_moe_forward_device on the same
 * expert path; with more ranks the fp32 sum is grouped by rank (within tolerance of the reference). */
int qe_moe_ep_route_device(QeMoe *m, int T, const float *x, int32_t *meta, float *shared, void *stream);
int qe_moe_ep_pack_device(QeMoe *m, int T, const float *x, const int32_t *meta, float *send_x, int32_t *send_meta,
                          int32_t *home, int32_t *counts, void *stream);
int qe_moe_ep_experts_device(QeMoe *m, int n, const float *x, const int32_t *meta, float *partial, void *stream);
int qe_moe_ep_combine_device(QeMoe *m, int T, const float *part, const int32_t *home, const float *shared, float *out,
                             void *stream);
int qe_moe_ep_size(const QeMoe *m);
/* Number of routed experts this handle holds; their global ids in slot order into ids (may be NULL). */
int qe_moe_ep_experts(const QeMoe *m, int32_t *ids);

/* Token-sharded step with the exchange done by the kernels themselves through peer memory (NVLink stores
 * into CUDA-IPC mappings of the other ranks' buffers), instead of two all_to_all calls:
 *   qe_ep_xchg_create        this rank's receive and return buffers for steps of up to T_max tokens per rank
 *                            (rows [G][T_max][h], slot lists [G][T_max][2k], partial rows [G][T_max][h]);
 *                            writes its qe_ep_xchg_handle_bytes()-byte IPC handle to `handle`
 *   qe_ep_xchg_connect       handles[G][handle bytes] of every rank (own entry ignored): map the peers
 *   qe_ep_xchg_connect_local ranks emulated in one process on one device (tests): n contexts, plain pointers
 * Per step, after qe_moe_ep_route_device:
 *   qe_moe_ep_dispatch_p2p   plan (home, counts as qe_moe_ep_pack_device) and write each row and slot list
 *                            into its destination rank's receive buffer (block = this rank, padded to T rows)
 *   (caller) a barrier across the ranks on the stream, e.g. a one-element all_reduce
 *   qe_moe_ep_experts_p2p    the expert stage on the G*T received rows, each partial row written into its
 *                            home rank's return buffer
 *   (caller) a barrier across the ranks on the stream
 *   qe_moe_ep_combine_p2p    out[t] = sum over ranks d ascending of return[d][home[d][t]] + shared[t]
 * Same arithmetic as the all_to_all step (bit-identical results). No multicast, only plain loads and stores.
 * Folded shared expert: routing the step with qe_moe_ep_route_p2p instead of qe_moe_ep_route_device computes
 * no shared term there; it copies the rank's own rows and shared-gate logits into the exchange, the expert
 * stage then runs the shared expert on them in the same launches as the received rows, and
 * qe_moe_ep_combine_p2p is called with shared = NULL (the term is read from the exchange). Same arithmetic
 * per token; the shared expert's batch is then the expert stage's, not the T own rows. Needs
 * T <= T_max and T <= the handle's max_tokens (and (G+1)*T <= max_tokens for one expert-stage pass). */
typedef struct QeEpXchg QeEpXchg;
QeEpXchg *qe_ep_xchg_create(QeMoe *m, int T_max, void *handle);
int qe_ep_xchg_handle_bytes(void);
int qe_ep_xchg_connect(QeEpXchg *x, const void *handles);
int qe_ep_xchg_connect_local(QeEpXchg *const *all, int n);
void qe_ep_xchg_free(QeEpXchg *x);
int qe_moe_ep_dispatch_p2p(QeMoe *m, QeEpXchg *xc, int T, const float *x, const int32_t *meta, int32_t *home,
                           int32_t *counts, void *stream);
/* A barrier across the ranks on the stream, in place of the caller's collective: every rank's work before it
 * on its stream (its stores into the peers' buffers included) is complete and visible before any rank's work
 * after it. One warp per rank publishes an epoch into each peer's flag slot and waits for every peer's, at
 * most 2 s; the epoch is a device counter, so the call can be captured in a CUDA graph and replayed. Every
 * rank must make the same sequence of calls, each on its own GPU (ranks emulated on one GPU must not use it:
 * a wait on a kernel of the same GPU may never end). A timeout is reported by qe_device_error() (200 + 1). */
int qe_ep_xchg_barrier(QeEpXchg *x, void *stream);
/* Bound of each wait in this context's qe_ep_xchg_barrier calls, 1 ms .. 60 s (default 2 s); a barrier launched
 * afterwards uses it (a CUDA graph keeps the bound it was captured with). 0 ok, -1 error. */
int qe_ep_xchg_set_timeout_ms(QeEpXchg *x, int ms);
int qe_moe_ep_route_p2p(QeMoe *m, QeEpXchg *xc, int T, const float *x, int32_t *meta, void *stream);
int qe_moe_ep_experts_p2p(QeMoe *m, QeEpXchg *xc, int T, void *stream);
int qe_moe_ep_combine_p2p(QeMoe *m, QeEpXchg *xc, int T, const int32_t *home, const float *shared, float *out,
                          void *stream);

/* Block accessors. */
int qe_moe_hidden(const QeMoe *m);
int qe_moe_top_k(const QeMoe *m);
size_t qe_moe_weight_bytes(const QeMoe *m);   /* HBM bytes held by this block's weights */

/* ---- kernel-level entry points (host buffers), the GPU counterparts of the reference's ops ---- */

/* y[rows] = W x, W one MLX-affine QMat (engine/include/qmat.h:32, engine/src/qmat.c:15-49). Same validation
 * as qmat_matvec: bits in {4,8}, group_size in {32,64,128}, rows > 0, cols > 0 and a multiple of
 * group_size, cols/group_size <= 4096; on error returns -1 and leaves y untouched. */
int qe_qmat_matvec(const uint32_t *w, const uint16_t *scales, const uint16_t *biases, int rows, int cols, int bits,
                   int group_size, const float *x, float *y);

/* T softmax + top-k + renormalisations on given logits[T][E] (engine/src/ops.c:29-73, moe_layer.c:31-36).
 * probs[T][E] (may be NULL), idx[T][k], score[T][k]. 1 <= k <= min(16, E), E <= 512. */
int qe_route_logits(int T, int E, int k, const float *logits, float *probs, int32_t *idx, float *score);

/* Element-wise ops of engine/src/ops.c:16-27 on the GPU (host buffers, n >= 1). */
int qe_op_silu_mul(float *out, const float *gate, const float *up, int n);
int qe_op_sigmoid(float *out, const float *x, int n);
/* The device expf used by softmax, on n inputs (for comparison with the host C library's expf). */
int qe_op_expf(float *out, const float *x, int n);

/* Routing (fp32 router, softmax, top-k, renormalisation) on device buffers without allocating any device
 * memory. No counterpart in the reference. It is for callers that cannot let a library call cudaMalloc:
 * a framework whose caching allocator already owns the device memory, or a decode loop that cannot take
 * the device-wide synchronisation an allocation may cause. router_w: device [E+1][hidden] fp32 (rows
 * 0..E-1 the router, row E the shared-expert gate vector, as qe_moe_create stores them); router_bias: device
 * [E] or NULL; x: device [T][hidden]; idx/score: device [T][top_k]; stream: a cudaStream_t (NULL = legacy
 * default). The only scratch, the logits, lives in a fixed 4 MiB device array (2^20 floats) that every GPU
 * loading the library holds until exit: T*(E+1) must not exceed 2^20 (T <= 4080 at E = 256), larger T is
 * refused with -1. All calls share that array, so calls that overlap on the GPU race. The first call on a
 * device looks up the array's device address, so make it before any stream capture. Same results as
 * qe_moe_route for the same weights. 0 ok, -1 error (message on stderr). */
int qe_route_f32_noalloc(const float *router_w, const float *router_bias, const float *x, int T, int hidden, int E,
                         int top_k, int32_t *idx, float *score, void *stream);

/* ---- engine-level statistics (engine/include/qengine.h:20-23 counterparts) ---- */
double qe_expert_gb_read(void);        /* GB of expert weights streamed from HBM by qe_moe_forward */
double qe_expert_read_seconds(void);   /* GPU seconds spent in qe_moe_forward's kernels            */
int qe_device_count(void);
/* Host threads the library uses from now on for its CPU-side work: paging a checkpoint's (or a host weight
 * array's) expert bytes in, in parallel, before they are copied to HBM (the GPU does the math). n <= 0 keeps
 * the current count. Returns the effective count (default: the host's hardware threads). Same signature and
 * return convention as the reference's qe_set_threads (engine/src/qengine.c:35-43, OpenMP threads there). */
int qe_set_threads(int n);
/* Peak resident set size of the process in GiB (getrusage; engine/src/qengine.c:47). Linux reports ru_maxrss
 * in KiB, macOS (the reference's platform) in bytes: the value here is converted from KiB. */
double qe_peak_rss_gb(void);

/* ---- profiling (no reference counterpart: the reference times only its expert reads, moe_layer.c:74-78) ---- */
enum { QE_STAGE_ROUTER = 0, QE_STAGE_TOPK, QE_STAGE_BUCKET, QE_STAGE_GATEUP, QE_STAGE_DOWN, QE_STAGE_COMBINE,
       QE_STAGES };
/* Record CUDA events around every stage of every forward pass on `device` from now on. */
int qe_profile_begin(int device);
/* Stop recording; stage_ms[QE_STAGES] = summed GPU milliseconds per stage, *passes = passes recorded. */
int qe_profile_end(int device, double *stage_ms, int *passes);
/* Kernels launched by this library since process start. */
unsigned long long qe_kernel_launches(void);
/* Forwards this library captured into CUDA graphs since process start (qe_moe_graph_create, and the graphs
 * qe_moe_forward_async captures for both staging slots on a handle's first call with a batch size). */
unsigned long long qe_graph_captures(void);
/* Nonzero if a bounded wait on the device timed out (the kernel then returned early; outputs invalid): a
 * tensor-core kernel's pipeline wait (its code), the fused decode step's grid barrier (100 + code), or the
 * exchange barrier of qe_ep_xchg_barrier (201). */
int qe_device_error(void);
/* qe_device_error for `device` (the caller's current device is left as it was). */
int qe_device_error_on(int device);
/* Clear every recorded timeout code on `device` (after the caller handled one). 0 ok, -1 error. */
int qe_device_error_reset(int device);

#ifdef __cplusplus
}
#endif
#endif
