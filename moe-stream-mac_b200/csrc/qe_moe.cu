/* qe_moe.cu: the C ABI of libqengine_b200 (include/qe_moe.h) and the block pipeline.
 *
 * Pipeline of one forward (replacing moe_layer_step, engine/src/moe_layer.c:66-89, for T tokens at once):
 *   1. router logits [T][E+1] (column E = shared-expert gate logit)          route.cu
 *   2. softmax + top-k + renormalise -> idx[T][k], score[T][k]                route.cu
 *   3. bucket (token, slot) pairs by expert, list the active experts         bucket.cu
 *   4. gate/up projections + SwiGLU for every (pair, expert) -> h3           expert_mma.cu
 *   5. down projection -> y per pair                                         expert_mma.cu
 *   6. out = sum_i score_i * y_i + sigmoid(gate logit) * y_shared           expert_mma.cu
 * The expert weights are resident in HBM for the handle's lifetime (the reference preads them from SSD
 * per token: engine/src/expert_store.c:54-61, moe_layer.c:42-55).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <atomic>
#include <mutex>
#include <thread>
#include <vector>
#include <sys/resource.h>

#include "qe_common.cuh"
#include "qe_kernels.h"
#include "synth.h"
#include "../../include/qe_moe.h"

int qe_expert_rows_per_cta(int T);

/* Expert path by batch size (auto): at most kDecodeMaxTokens tokens take the decode GEMVs (decode.cu); larger
 * batches with at most kGroupMaxPerExpert routed assignments per expert on average the grouped GEMVs
 * (group_gemv.cu: measured faster than the tcgen05 kernels from 8 to 128 tokens on the 4-bit and 8-bit benchmark
 * blocks, E=256, top-8); larger batches the tensor-core (tcgen05) kernels when the shape allows; shapes neither
 * covers take the mma.sync kernels. QE_EXPERT_PATH=mma|tc|gemv|group forces one. */
static constexpr int kTcMinTokens = 5;
static constexpr int kDecodeMaxTokens = 4;
static constexpr int kGroupMaxPerExpert = 4;

/* ------------------------------------------------------------------ per-device context and workspace */

namespace {

struct DevCtx {
    bool init = false;
    cudaStream_t stream = nullptr;
    int sms = 0;
    void *ws = nullptr;       /* scratch workspace shared by all handles on this device */
    size_t ws_bytes = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    /* pipelined host-buffer forwards (qe_moe_forward_async): copy-in and copy-out streams and two staging
     * slots, each an x and an out buffer of stage_cap floats */
    cudaStream_t s_in = nullptr, s_out = nullptr;
    float *stage = nullptr;
    size_t stage_cap = 0;
    cudaEvent_t ev_h2d[2] = {}, ev_comp[2] = {}, ev_d2h[2] = {};
    bool slot_used[2] = {false, false};
    unsigned long long async_n = 0;
};

std::mutex g_mu;
DevCtx g_dev[64];
std::atomic<unsigned long long> g_bytes_read{0};
std::atomic<int> g_host_threads{0};   /* qe_set_threads; 0 = the host's hardware threads */

int host_threads() {
    const int n = g_host_threads.load();
    if (n > 0) return n;
    const unsigned hw = std::thread::hardware_concurrency();
    return hw ? (int)hw : 1;
}

/* Touch one byte per 4 KiB page of [p, p + bytes) on the library's host threads, so that a memory-mapped
 * checkpoint is read from the file in parallel before the (single-threaded) copy to HBM walks it. */
void page_in(const void *p, size_t bytes) {
    constexpr size_t kPage = 4096, kMinPerThread = 8u << 20;
    const int nt = (int)std::min<size_t>((size_t)host_threads(), std::max<size_t>(1, bytes / kMinPerThread));
    const char *c = (const char *)p;
    auto touch = [c](size_t a, size_t b) {
        unsigned sum = 0;
        for (size_t o = a; o < b; o += kPage) sum += (unsigned char)((const volatile char *)c)[o];
        if (b > a) sum += (unsigned char)((const volatile char *)c)[b - 1];
        (void)sum;
    };
    if (nt <= 1) {
        touch(0, bytes);
        return;
    }
    std::vector<std::thread> pool;
    const size_t per = (bytes / nt + kPage - 1) / kPage * kPage;
    for (int i = 0; i < nt; i++) {
        const size_t a = std::min(bytes, (size_t)i * per), b = std::min(bytes, a + per);
        if (a < b) pool.emplace_back(touch, a, b);
    }
    for (auto &t : pool) t.join();
}
double g_gpu_seconds = 0.0;
std::atomic<unsigned long long> g_launches{0};
std::atomic<unsigned long long> g_captures{0};   /* forwards captured into CUDA graphs */

/* Stage profiling: when enabled, every pass records one event before the router and one after each of
 * the QE_STAGES stages on the stream it runs on; qe_profile_end sums the per-stage elapsed times. */
constexpr int kStages = 6;
struct Prof {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
};
Prof g_prof[64];

cudaEvent_t prof_event(int dev) {
    Prof &p = g_prof[dev];
    if (p.used == p.pool.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
        p.pool.push_back(e);
    }
    return p.pool[p.used++];
}

void prof_mark(int dev, cudaStream_t s) {
    if (!g_prof[dev].on) return;
    cudaEvent_t e = prof_event(dev);
    if (e) cudaEventRecord(e, s);
}

int dev_ctx(int device, DevCtx **out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) QE_FAIL("no CUDA device available");
    if (device < 0 || device >= n || device >= 64) QE_FAIL("device %d out of range (%d devices)", device, n);
    QE_CHECK(cudaSetDevice(device));
    DevCtx &d = g_dev[device];
    if (!d.init) {
        int major = 0;
        QE_CHECK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        if (major != 10) QE_FAIL("device %d has compute capability %d.x; this library is built for sm_100a", device, major);
        QE_CHECK(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device));
        QE_CHECK(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
        QE_CHECK(cudaEventCreate(&d.ev0));
        QE_CHECK(cudaEventCreate(&d.ev1));
        d.init = true;
    }
    *out = &d;
    return 0;
}

int ensure_ws(DevCtx *d, size_t bytes) {
    if (d->ws_bytes >= bytes) return 0;
    if (d->ws) {
        QE_CHECK(cudaStreamSynchronize(d->stream));
        QE_CHECK(cudaDeviceSynchronize());
        cudaFree(d->ws);
        d->ws = nullptr;
        d->ws_bytes = 0;
    }
    QE_CHECK(cudaMalloc(&d->ws, bytes));
    d->ws_bytes = bytes;
    return 0;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

/* Carves a workspace into the per-forward buffers. */
struct Scratch {
    float *x, *out, *logits, *score, *h3, *ybuf;
    float *rpart;               /* fp32 router chunk values [hidden/64][T][E+1] (prefill GEMM) */
    float *rxt;                 /* the batch transposed for the prefill router GEMM, [hidden][T rounded up to 4] */
    int32_t *idx;
    QeBuckets b;
    QeTcBufs tcb;               /* tensor-core path: split activations, group sums, unscale factors */
    unsigned *gbar;             /* grid barrier of the fused decode kernel */
};

size_t scratch_layout(const QeMoeConfig &c, int T, char *base, Scratch *s) {
    const int E = c.E, k = c.top_k, I = c.inter > c.sh_inter ? c.inter : c.sh_inter;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char * {
        char *p = base ? base + off : nullptr;
        off += align256(bytes);
        return p;
    };
    const size_t npair = (size_t)T * (k + 1);
    Scratch t;
    t.x = (float *)take(sizeof(float) * (size_t)T * c.hidden);
    t.out = (float *)take(sizeof(float) * (size_t)T * c.hidden);
    t.logits = (float *)take(sizeof(float) * (size_t)T * (E + 1));
    t.rpart = (float *)take(sizeof(float) * (size_t)((c.hidden + 63) / 64) * T * (E + 1));
    t.rxt = (float *)take(sizeof(float) * (size_t)c.hidden * ((T + 3) & ~3));
    t.score = (float *)take(sizeof(float) * (size_t)T * k);
    t.idx = (int32_t *)take(sizeof(int32_t) * (size_t)T * k);
    t.h3 = (float *)take(sizeof(float) * npair * I);
    t.ybuf = (float *)take(sizeof(float) * npair * c.hidden);
    t.b.counts = (int32_t *)take(sizeof(int32_t) * (E + 1));
    t.b.offsets = (int32_t *)take(sizeof(int32_t) * (E + 2));
    t.b.cursor = (int32_t *)take(sizeof(int32_t) * (E + 1));
    t.b.pairs = (int32_t *)take(sizeof(int32_t) * npair);
    t.b.slot_expert = (int32_t *)take(sizeof(int32_t) * (E + 2));
    t.b.slot_items = (int32_t *)take(sizeof(int32_t) * 2 * (E + 2));
    t.b.n_active = (int32_t *)take(sizeof(int32_t) * 4);
    t.b.chunks = (int4 *)take(sizeof(int4) * npair);
    t.tcb.act = (__half *)take(2 * 2 * (size_t)T * c.hidden);
    t.tcb.actsum = (float *)take(4 * (size_t)T * (c.hidden / 64 + 1));
    t.tcb.actinv = (float *)take(4 * (size_t)T * (c.hidden / 64 + 1));
    t.tcb.h3s = (__half *)take(2 * 2 * npair * I);
    t.tcb.h3sum = (float *)take(4 * npair * (I / 64 + 1));
    t.tcb.h3inv = (float *)take(4 * npair * (I / 64 + 1));
    t.tcb.ldh = I;
    t.gbar = (unsigned *)take(2 * sizeof(unsigned));
    if (s) *s = t;
    return off;
}

}  // namespace

/* ------------------------------------------------------------------ handle */

struct QeMoe {
    QeMoeConfig cfg;
    int device;
    void *weights;          /* one HBM allocation holding every tensor of the block */
    size_t weight_bytes;
    float *router_w;        /* [E+1][H] (F32 mode; row E = shared gate) */
    float *router_wd;       /* [H][qe_router_wd_rows(E)][2]: router_w duplicated for the prefill GEMM (F32 mode) */
    float *router_bias;     /* [E] or null */
    QeQDev router_q, sh_router_q;
    QeExpertArgs ex;
    size_t expert_bytes;    /* bytes of one routed expert (gate+up+down codes, scales, biases) */
    int e0, E_loc;          /* routed experts held here: E_loc of them, global ids held[0 .. E_loc) in slot order
                             * ([e0, e0 + E_loc) without a placement table; e0 = -1 with one) */
    int32_t held[512];
    int32_t *place;         /* device [E][2 + ep_size]: local slot of e here (-1: not held), replica count, the
                             * holding ranks ascending (expert parallelism) */
    int path;               /* 0 = auto, 1 = mma.sync, 2 = tensor-core (tcgen05), 3 = decode GEMVs, 4 = grouped GEMVs */
    bool tc;                /* tensor-core path available for this shape */
    bool decode;            /* decode GEMVs available for this shape */
    bool group;             /* grouped GEMVs available for this shape */
    int tile;               /* tensor-core token tile: 0 = by load, else 32 or 64 (QE_TC_TILE) */
    QeMoeGraph *agraph[2];  /* qe_moe_forward_async: the forward captured per staging slot, for a_T, a_x, a_o */
    int a_T[2];
    const float *a_x[2], *a_o[2];
    bool fused;             /* decode steps as one cooperative launch (QE_DECODE_FUSED=1; measured slower than
                             * the four launches replayed from a CUDA graph, so off by default) */
    alignas(64) unsigned char maps_gu[2 * 2 * 3 * 128];  /* [routed/shared][gate/up][codes, scales, biases] */
    alignas(64) unsigned char maps_dn[2 * 3 * 128];      /* [routed/shared][codes, scales, biases] */
};

namespace {

int validate(const QeMoeConfig *c) {
    if (!c) QE_FAIL("null config");
    if (c->top_k < 1 || c->top_k > 16) QE_FAIL("top_k=%d outside [1, 16] (MOE_MAX_TOPK)", c->top_k);
    if (c->E < c->top_k || c->E > 512) QE_FAIL("E=%d outside [top_k, 512]", c->E);
    if (c->bits != 4 && c->bits != 8) QE_FAIL("bits=%d: only 4 and 8 are supported", c->bits);
    if (c->group_size != 32 && c->group_size != 64 && c->group_size != 128)
        QE_FAIL("group_size=%d: only 32, 64 and 128 are supported", c->group_size);
    if (c->hidden <= 0 || c->inter <= 0 || c->sh_inter <= 0) QE_FAIL("non-positive dimension");
    if (c->hidden % c->group_size || c->inter % c->group_size || c->sh_inter % c->group_size)
        QE_FAIL("hidden/inter/sh_inter must be multiples of group_size %d", c->group_size);
    if (c->hidden > 8192) QE_FAIL("hidden=%d > 8192", c->hidden);
    if (c->router_mode != QE_ROUTER_F32 && c->router_mode != QE_ROUTER_QMAT) QE_FAIL("bad router_mode");
    if (c->router_mode == QE_ROUTER_QMAT && c->router_bits != 4 && c->router_bits != 8)
        QE_FAIL("router_bits=%d: only 4 and 8", c->router_bits);
    const int G = c->ep_size < 1 ? 1 : c->ep_size;
    if (G > 64) QE_FAIL("ep_size=%d above 64", c->ep_size);
    if (c->ep_rank < 0 || c->ep_rank >= G) QE_FAIL("ep_rank=%d outside [0, %d)", c->ep_rank, G);
    if (!c->placement) {
        if (c->E % G) QE_FAIL("ep_size=%d must divide E=%d (or give a placement)", c->ep_size, c->E);
        return 0;
    }
    if (G < 2) QE_FAIL("a placement needs ep_size > 1");
    if (c->slots < 1 || c->slots > c->E) QE_FAIL("placement: slots=%d outside [1, E=%d]", c->slots, c->E);
    std::vector<int> seen(c->E, 0), row(c->E, -1);
    for (int r = 0; r < G; r++) {
        int n = 0;
        for (int j = 0; j < c->slots; j++) {
            const int e = c->placement[(size_t)r * c->slots + j];
            if (e == -1) continue;
            if (e < 0 || e >= c->E) QE_FAIL("placement[%d][%d] = %d is not an expert id", r, j, e);
            if (row[e] == r) QE_FAIL("placement: rank %d lists expert %d twice", r, e);
            row[e] = r;
            seen[e]++;
            n++;
        }
        if (!n) QE_FAIL("placement: rank %d holds no expert", r);
    }
    for (int e = 0; e < c->E; e++)
        if (!seen[e]) QE_FAIL("placement: expert %d is held by no rank", e);
    return 0;
}

/* The device placement table of a handle, [E][2 + G] int32: per expert its local slot on `rank` (-1 if not held
 * there), its replica count and the ranks holding it, ascending (-1 past the count). */
std::vector<int32_t> placement_table(const QeMoeConfig *c, int G, int rank, int32_t *held, int *n_held) {
    const int E = c->E, W = 2 + G;
    std::vector<int32_t> t((size_t)E * W, -1);
    for (int e = 0; e < E; e++) t[(size_t)e * W + 1] = 0;
    *n_held = 0;
    for (int r = 0; r < G; r++) {
        const int S = c->placement ? c->slots : E / G;
        for (int j = 0; j < S; j++) {
            const int e = c->placement ? c->placement[(size_t)r * S + j] : r * S + j;
            if (e < 0) continue;
            int32_t *te = &t[(size_t)e * W];
            te[2 + te[1]++] = r;
            if (r == rank) {
                te[0] = *n_held;
                held[(*n_held)++] = e;
            }
        }
    }
    return t;
}

size_t qbytes(int n, int rows, int cols, int bits, int gs, size_t *wb, size_t *gb) {
    *wb = (size_t)n * rows * ((size_t)cols * bits / 32) * 4;
    *gb = (size_t)n * rows * ((size_t)cols / gs) * 2;
    return *wb + 2 * *gb;
}

/* Allocate the handle and carve its HBM block. */
QeMoe *alloc_handle(const QeMoeConfig *c) {
    if (validate(c)) return nullptr;
    DevCtx *d;
    if (dev_ctx(c->device, &d)) return nullptr;
    QeMoe *m = (QeMoe *)aligned_alloc(64, (sizeof(QeMoe) + 63) & ~(size_t)63);
    if (!m) return nullptr;
    memset(m, 0, sizeof(QeMoe));
    m->cfg = *c;
    if (m->cfg.max_tokens < 1) m->cfg.max_tokens = 4096;
    if (m->cfg.ep_size < 1) m->cfg.ep_size = 1;
    m->device = c->device;
    const int G = m->cfg.ep_size;
    const std::vector<int32_t> table = placement_table(&m->cfg, G, m->cfg.ep_rank, m->held, &m->E_loc);
    m->e0 = c->placement ? -1 : m->cfg.ep_rank * m->E_loc;
    m->cfg.placement = nullptr;   /* the caller's table is not kept */
    const int E = c->E, El = m->E_loc, H = c->hidden, I = c->inter, Is = c->sh_inter, b = c->bits,
              gs = c->group_size;
    struct Part { int n, rows, cols, bits; QeQDev *dst; };
    Part parts[8] = {
        {El, I, H, b, &m->ex.gate}, {El, I, H, b, &m->ex.up}, {El, H, I, b, &m->ex.down},
        {1, Is, H, b, &m->ex.sh_gate}, {1, Is, H, b, &m->ex.sh_up}, {1, H, Is, b, &m->ex.sh_down},
        {c->router_mode == QE_ROUTER_QMAT ? 1 : 0, E, H, c->router_bits, &m->router_q},
        {c->router_mode == QE_ROUTER_QMAT ? 1 : 0, 1, H, c->router_bits, &m->sh_router_q}};
    size_t total = 0;
    for (auto &p : parts) {
        if (!p.n) continue;
        size_t wb, gb;
        qbytes(p.n, p.rows, p.cols, p.bits, gs, &wb, &gb);
        total += align256(wb) + 2 * align256(gb);
    }
    const size_t wd_bytes = sizeof(float) * 2 * (size_t)H * qe_router_wd_rows(E);
    if (c->router_mode == QE_ROUTER_F32)
        total += align256(sizeof(float) * (size_t)(E + 1) * H) + align256(4 * (size_t)E) + align256(wd_bytes);
    const size_t table_bytes = sizeof(int32_t) * table.size();
    total += align256(table_bytes);
    char *base = nullptr;
    if (cudaMalloc((void **)&base, total) != cudaSuccess) {
        fprintf(stderr, "qengine_b200: cannot allocate %zu bytes of HBM for the block\n", total);
        free(m);
        return nullptr;
    }
    m->weights = base;
    m->weight_bytes = total;
    size_t off = 0;
    for (auto &p : parts) {
        if (!p.n) continue;
        size_t wb, gb;
        qbytes(p.n, p.rows, p.cols, p.bits, gs, &wb, &gb);
        p.dst->w = (const uint32_t *)(base + off); off += align256(wb);
        p.dst->scales = (const uint16_t *)(base + off); off += align256(gb);
        p.dst->biases = (const uint16_t *)(base + off); off += align256(gb);
        p.dst->rows = p.rows; p.dst->cols = p.cols; p.dst->bits = p.bits; p.dst->group_size = gs;
        p.dst->scale_t = (&p - parts) < 6;   /* expert tensors keep scales/biases as [n][groups][rows] */
    }
    if (c->router_mode == QE_ROUTER_F32) {
        m->router_w = (float *)(base + off); off += align256(sizeof(float) * (size_t)(E + 1) * H);
        m->router_bias = (float *)(base + off); off += align256(4 * (size_t)E);
        m->router_wd = (float *)(base + off); off += align256(wd_bytes);
    }
    m->place = (int32_t *)(base + off); off += align256(table_bytes);
    if (cudaMemcpy(m->place, table.data(), table_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        fprintf(stderr, "qengine_b200: cannot copy the placement table\n");
        cudaFree(base);
        free(m);
        return nullptr;
    }
    m->ex.E = El; m->ex.k = c->top_k; m->ex.hidden = H; m->ex.inter = I; m->ex.sh_inter = Is;
    size_t wb, gb;
    m->expert_bytes = qbytes(1, I, H, b, gs, &wb, &gb) * 2 + qbytes(1, H, I, b, gs, &wb, &gb);
    const char *path = getenv("QE_EXPERT_PATH");   /* auto (default) | mma | tc | gemv | group */
    m->path = path && !strcmp(path, "mma") ? 1 : path && !strcmp(path, "tc") ? 2 : path && !strcmp(path, "gemv") ? 3
            : path && !strcmp(path, "group") ? 4 : 0;
    m->group = qe_group_supported(&m->ex);
    const char *fz = getenv("QE_DECODE_FUSED");
    m->fused = fz && !strcmp(fz, "1");
    const char *tt = getenv("QE_TC_TILE");
    m->tile = tt && !strcmp(tt, "32") ? 32 : tt && !strcmp(tt, "64") ? 64 : 0;
    m->tc = qe_tc_supported(&m->ex);
    m->decode = qe_decode_supported(&m->ex);
    if (m->tc) {
        const size_t mb = qe_tc_map_bytes();
        const QeQDev *gu[2][2] = {{&m->ex.gate, &m->ex.up}, {&m->ex.sh_gate, &m->ex.sh_up}};
        const QeQDev *dn[2] = {&m->ex.down, &m->ex.sh_down};
        for (int r = 0; r < 2 && m->tc; r++) {
            for (int q = 0; q < 2 && m->tc; q++) {
                unsigned char *o = m->maps_gu + ((r * 2 + q) * 3) * mb;
                m->tc = !qe_tc_weight_maps(gu[r][q], r ? 1 : El, o, o + mb, o + 2 * mb);
            }
            unsigned char *o = m->maps_dn + (r * 3) * mb;
            if (m->tc) m->tc = !qe_tc_weight_maps(dn[r], r ? 1 : El, o, o + mb, o + 2 * mb);
        }
    }
    return m;
}

/* The routed-expert tensor q from local slot `slot` on (each expert's codes and its scales/biases are contiguous
 * in both scale layouts). */
QeQDev at_slot(const QeQDev &q, int slot) {
    QeQDev r = q;
    const size_t wpm = (size_t)q.rows * ((size_t)q.cols * q.bits / 32), gpm = (size_t)q.rows * (q.cols / q.group_size);
    r.w += (size_t)slot * wpm;
    r.scales += (size_t)slot * gpm;
    r.biases += (size_t)slot * gpm;
    return r;
}

/* f(slot, first, n) for each maximal run of local slots holding consecutive global ids first .. first + n - 1
 * (one run for a contiguous range); stops at the first nonzero result. */
template <class F>
int for_runs(const QeMoe *m, F f) {
    for (int j = 0; j < m->E_loc;) {
        int n = 1;
        while (j + n < m->E_loc && m->held[j + n] == m->held[j] + n) n++;
        if (int rc = f(j, m->held[j], n)) return rc;
        j += n;
    }
    return 0;
}

/* Copies matrices [first, first + n) of a host tensor into dst. */
int upload_q(const QeQDev *dst, const QeQTensor *src0, int n, cudaStream_t s, int first = 0) {
    if (!src0->w || !src0->scales || !src0->biases) QE_FAIL("missing quantized tensor");
    const int ng = dst->cols / dst->group_size;
    const size_t wpm = (size_t)dst->rows * ((size_t)dst->cols * dst->bits / 32), gpm = (size_t)dst->rows * ng;
    QeQTensor src1 = {src0->w + (size_t)first * wpm, src0->scales + (size_t)first * gpm,
                      src0->biases + (size_t)first * gpm};
    const QeQTensor *src = &src1;
    const size_t wb = (size_t)n * dst->rows * ((size_t)dst->cols * dst->bits / 32) * 4;
    const size_t gb = (size_t)n * dst->rows * (size_t)ng * 2;
    page_in(src->w, wb);
    page_in(src->scales, gb);
    page_in(src->biases, gb);
    QE_CHECK(cudaMemcpyAsync((void *)dst->w, src->w, wb, cudaMemcpyHostToDevice, s));
    if (!dst->scale_t) {
        QE_CHECK(cudaMemcpyAsync((void *)dst->scales, src->scales, gb, cudaMemcpyHostToDevice, s));
        QE_CHECK(cudaMemcpyAsync((void *)dst->biases, src->biases, gb, cudaMemcpyHostToDevice, s));
        return 0;
    }
    /* MLX [n][rows][groups] in, [n][groups][rows] resident: a reversible transpose on the device */
    uint16_t *tmp = nullptr;
    QE_CHECK(cudaMalloc((void **)&tmp, gb));
    int rc = cudaMemcpyAsync(tmp, src->scales, gb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
             qe_launch_transpose_groups(tmp, (uint16_t *)dst->scales, n, dst->rows, ng, s) ||
             cudaMemcpyAsync(tmp, src->biases, gb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
             qe_launch_transpose_groups(tmp, (uint16_t *)dst->biases, n, dst->rows, ng, s) ||
             cudaStreamSynchronize(s) != cudaSuccess;
    cudaFree(tmp);
    if (rc) QE_FAIL("scale upload failed");
    return 0;
}

/* Scale/bias i is generated from its MLX-order index (n, row, group) so the values match the CPU
 * checker's copy; with scale_t it is stored at [n][group][row]. word0/group0: index of the first generated
 * element in the whole tensor (an expert-parallel handle generates only its own experts' slice). */
__global__ void synth_qmat_kernel(uint64_t seed, uint32_t block, uint32_t stream, size_t word0, size_t group0,
                                  size_t nwords, size_t ngroups, int rows, int ng, int scale_t, float scale_c,
                                  float neg_half, uint32_t *w, uint16_t *sc, uint16_t *bi) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords; i += stride)
        w[i] = syn_code_word(seed, block, stream, word0 + i);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < ngroups; i += stride) {
        uint16_t s, b;
        syn_scale_bias(seed, block, stream, group0 + i, scale_c, neg_half, &s, &b);
        size_t o = i;
        if (scale_t) {
            const size_t e = i / ((size_t)rows * ng), r = (i / ng) % rows, g = i % ng;
            o = (e * ng + g) * rows + r;
        }
        sc[o] = s;
        bi[o] = b;
    }
}

__global__ void transpose_groups_kernel(const uint16_t *__restrict__ src, uint16_t *__restrict__ dst, int rows,
                                        int ng, size_t total) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const size_t e = i / ((size_t)rows * ng), r = (i / ng) % rows, g = i % ng;
        dst[(e * ng + g) * rows + r] = src[i];
    }
}

__global__ void synth_normal_kernel(uint64_t seed, uint32_t block, uint32_t stream, size_t n, float sigma_c,
                                    float *out) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = syn_normal(syn_hash(seed, block, stream, i), sigma_c);
}

__global__ void ops_kernel(int op, const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
                           int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (op == 0) out[i] = qe_silu_mul(a[i], b[i]);
    else if (op == 1) out[i] = qe_sigmoid(a[i]);
    else out[i] = qe_expf(a[i]);
}

}  // namespace

int qe_launch_synth_qmat(uint64_t seed, uint32_t block, uint32_t stream, int first, int n, int rows, int cols,
                         int bits, int gs, int scale_t, uint32_t *w, uint16_t *sc, uint16_t *bi, cudaStream_t s) {
    const size_t wpm = (size_t)rows * ((size_t)cols * bits / 32), gpm = (size_t)rows * (cols / gs);
    synth_qmat_kernel<<<1184, 256, 0, s>>>(seed, block, stream, (size_t)first * wpm, (size_t)first * gpm,
                                           (size_t)n * wpm, (size_t)n * gpm, rows, cols / gs, scale_t,
                                           syn_scale_c(bits), syn_neg_half_range(bits), w, sc, bi);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_transpose_groups(const uint16_t *src, uint16_t *dst, int n, int rows, int groups, cudaStream_t s) {
    transpose_groups_kernel<<<592, 256, 0, s>>>(src, dst, rows, groups, (size_t)n * rows * groups);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_launch_synth_normal(uint64_t seed, uint32_t block, uint32_t stream, size_t n, float sigma_c, float *out,
                           cudaStream_t s) {
    synth_normal_kernel<<<592, 256, 0, s>>>(seed, block, stream, n, sigma_c, out);
    QE_CHECK(cudaGetLastError());
    return 0;
}

int qe_num_sms(void) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

extern "C" {

QeMoe *qe_moe_create(const QeMoeConfig *cfg, const QeMoeWeights *w) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!w) { fprintf(stderr, "qengine_b200: null weights\n"); return nullptr; }
    QeMoe *m = alloc_handle(cfg);
    if (!m) return nullptr;
    DevCtx *d = &g_dev[m->device];
    cudaStream_t s = d->stream;
    int rc = for_runs(m, [&](int slot, int first, int n) {
                 const QeQDev g = at_slot(m->ex.gate, slot), u = at_slot(m->ex.up, slot), dn = at_slot(m->ex.down, slot);
                 return upload_q(&g, &w->gate, n, s, first) || upload_q(&u, &w->up, n, s, first) ||
                        upload_q(&dn, &w->down, n, s, first);
             }) ||
             upload_q(&m->ex.sh_gate, &w->sh_gate, 1, s) || upload_q(&m->ex.sh_up, &w->sh_up, 1, s) ||
             upload_q(&m->ex.sh_down, &w->sh_down, 1, s);
    if (!rc && cfg->router_mode == QE_ROUTER_QMAT)
        rc = upload_q(&m->router_q, &w->router_q, 1, s) || upload_q(&m->sh_router_q, &w->sh_router_q, 1, s);
    if (!rc && cfg->router_mode == QE_ROUTER_F32) {
        if (!w->router_f32 || !w->sh_gate_f32) {
            fprintf(stderr, "qengine_b200: fp32 router mode needs router_f32 and sh_gate_f32\n");
            rc = -1;
        } else {
            const size_t H = cfg->hidden, E = cfg->E;
            rc = cudaMemcpyAsync(m->router_w, w->router_f32, 4 * E * H, cudaMemcpyHostToDevice, s) != cudaSuccess ||
                 cudaMemcpyAsync(m->router_w + E * H, w->sh_gate_f32, 4 * H, cudaMemcpyHostToDevice, s) != cudaSuccess;
            if (!rc) rc = qe_launch_router_wd_fill(m->router_w, (int)H, (int)E, m->router_wd, s);
            if (!rc && w->router_bias)
                rc = cudaMemcpyAsync(m->router_bias, w->router_bias, 4 * E, cudaMemcpyHostToDevice, s) != cudaSuccess;
            if (!w->router_bias) m->router_bias = nullptr;
        }
    }
    if (!rc) rc = cudaStreamSynchronize(s) != cudaSuccess;
    if (rc) {
        fprintf(stderr, "qengine_b200: weight upload failed\n");
        cudaFree(m->weights);
        free(m);
        return nullptr;
    }
    return m;
}

QeMoe *qe_moe_create_synthetic(const QeMoeConfig *cfg, uint64_t seed, uint32_t block, const float *router_bias) {
    std::lock_guard<std::mutex> lock(g_mu);
    QeMoe *m = alloc_handle(cfg);
    if (!m) return nullptr;
    cudaStream_t s = g_dev[m->device].stream;
    const int E = cfg->E, H = cfg->hidden, I = cfg->inter, Is = cfg->sh_inter, b = cfg->bits, gs = cfg->group_size;
    auto gen = [&](const QeQDev &q, uint32_t stream, int n, int first = 0) {
        return qe_launch_synth_qmat(seed, block, stream, first, n, q.rows, q.cols, q.bits, gs, q.scale_t,
                                    (uint32_t *)q.w, (uint16_t *)q.scales, (uint16_t *)q.biases, s);
    };
    int rc = for_runs(m, [&](int slot, int first, int n) {
                 return gen(at_slot(m->ex.gate, slot), SYN_GATE, n, first) ||
                        gen(at_slot(m->ex.up, slot), SYN_UP, n, first) ||
                        gen(at_slot(m->ex.down, slot), SYN_DOWN, n, first);
             }) ||
             gen(m->ex.sh_gate, SYN_SH_GATE, 1) || gen(m->ex.sh_up, SYN_SH_UP, 1) || gen(m->ex.sh_down, SYN_SH_DOWN, 1);
    (void)I; (void)Is; (void)b;
    if (!rc && cfg->router_mode == QE_ROUTER_QMAT)
        rc = gen(m->router_q, SYN_ROUTER, 1) || gen(m->sh_router_q, SYN_SHGATE, 1);
    if (!rc && cfg->router_mode == QE_ROUTER_F32) {
        const float c = syn_sigma_c(0.02);
        rc = qe_launch_synth_normal(seed, block, SYN_ROUTER, (size_t)E * H, c, m->router_w, s) ||
             qe_launch_synth_normal(seed, block, SYN_SHGATE, (size_t)H, c, m->router_w + (size_t)E * H, s) ||
             qe_launch_router_wd_fill(m->router_w, H, E, m->router_wd, s);
        if (!rc && router_bias)
            rc = cudaMemcpyAsync(m->router_bias, router_bias, 4 * (size_t)E, cudaMemcpyHostToDevice, s) != cudaSuccess;
        if (!router_bias) m->router_bias = nullptr;
    }
    if (!rc) rc = cudaStreamSynchronize(s) != cudaSuccess;
    if (rc) {
        fprintf(stderr, "qengine_b200: synthetic block generation failed\n");
        cudaFree(m->weights);
        free(m);
        return nullptr;
    }
    return m;
}

void qe_moe_free(QeMoe *m) {
    if (!m) return;
    std::lock_guard<std::mutex> lock(g_mu);
    cudaSetDevice(m->device);
    cudaStreamSynchronize(g_dev[m->device].stream);
    if (g_dev[m->device].s_out) cudaStreamSynchronize(g_dev[m->device].s_out);
    for (int j = 0; j < 2; j++) qe_moe_graph_free(m->agraph[j]);
    cudaFree(m->weights);
    free(m);
}

int qe_moe_hidden(const QeMoe *m) { return m ? m->cfg.hidden : -1; }
int qe_moe_top_k(const QeMoe *m) { return m ? m->cfg.top_k : -1; }
size_t qe_moe_weight_bytes(const QeMoe *m) { return m ? m->weight_bytes : 0; }

}  // extern "C"

namespace {

/* The grouped GEMVs take a pass of T rows when selected (QE_EXPERT_PATH=group), or automatically when its routed
 * assignments average at most kGroupMaxPerExpert per expert: there the expert stage is the weight stream, and the
 * tensor-core tiles would spend a 32-token tile's conversion and epilogue on a few tokens. */
bool group_path(const QeMoe *m, int T) {
    if (!m->group) return false;
    if (m->path == 4) return true;
    return m->path == 0 && T > kDecodeMaxTokens &&
           (long long)T * m->cfg.top_k <= (long long)kGroupMaxPerExpert * m->cfg.E;
}

/* Routing for one pass of T tokens: logits + idx/score in the scratch. */
int run_route(QeMoe *m, const float *x, int T, Scratch &sc, cudaStream_t s) {
    const QeMoeConfig &c = m->cfg;
    if (c.router_mode == QE_ROUTER_F32) {
        const int nr = qe_launch_router_f32(m->router_w, m->router_bias, x, T, c.hidden, c.E, sc.logits, sc.rpart,
                                            m->router_wd, sc.rxt, s);
        if (nr < 0) return -1;
        g_launches += nr;
    } else {
        if (qe_launch_router_qmat(&m->router_q, &m->sh_router_q, x, T, c.hidden, c.E, sc.logits, s)) return -1;
        g_launches += 2;
    }
    if (qe_launch_route_topk(sc.logits, c.E + 1, T, c.E, c.top_k, sc.idx, sc.score, nullptr, s)) return -1;
    g_launches += 1;
    return 0;
}

int run_pass(QeMoe *m, const float *x, float *out, int T, Scratch &sc, int sms, cudaStream_t s) {
    const QeMoeConfig &c = m->cfg;
    const int dev = m->device;
    prof_mark(dev, s);
    const bool decode = m->decode && (m->path == 3 || (m->path == 0 && T <= kDecodeMaxTokens));
    if (decode && m->fused && c.router_mode == QE_ROUTER_F32) {
        /* the whole step as one cooperative launch (router, top-k, gate/up, down + combine); its time is
         * recorded as the router stage, the other stages are empty */
        const int I = c.inter > c.sh_inter ? c.inter : c.sh_inter;
        const int r = qe_launch_decode_fused(&m->ex, m->router_w, m->router_bias, x, T, sc.logits, sc.idx, sc.score,
                                             sc.h3, I, out, sc.gbar, sms, s);
        if (r < 0) return -1;
        if (r == 0) {
            for (int i = 0; i < 6; i++) prof_mark(dev, s);
            g_launches += 1;
            return 0;
        }
    }
    if (c.router_mode == QE_ROUTER_F32) {
        const int nr = qe_launch_router_f32(m->router_w, m->router_bias, x, T, c.hidden, c.E, sc.logits, sc.rpart,
                                            m->router_wd, sc.rxt, s);
        if (nr < 0) return -1;
        g_launches += nr;
    } else {
        if (qe_launch_router_qmat(&m->router_q, &m->sh_router_q, x, T, c.hidden, c.E, sc.logits, s)) return -1;
        g_launches += 2;
    }
    prof_mark(dev, s);
    if (qe_launch_route_topk(sc.logits, c.E + 1, T, c.E, c.top_k, sc.idx, sc.score, nullptr, s)) return -1;
    g_launches += 1;
    prof_mark(dev, s);
    const int I = c.inter > c.sh_inter ? c.inter : c.sh_inter;
    if (decode) {
        /* decode: CUDA-core GEMVs over each selected expert's codes, combine fused into the down projection */
        prof_mark(dev, s);   /* no bucketing */
        if (qe_launch_decode_gateup(&m->ex, x, sc.idx, T, sc.h3, I, s)) return -1;
        prof_mark(dev, s);
        if (qe_launch_decode_down_combine(&m->ex, sc.h3, I, sc.idx, sc.score, sc.logits, c.E + 1, T, out, s))
            return -1;
        prof_mark(dev, s);
        prof_mark(dev, s);   /* combine: fused into down */
        g_launches += 2;
        return 0;
    }
    const bool use_group = group_path(m, T);
    if (use_group) {
        /* batched decode: every active expert's rows streamed once per chunk of its tokens */
        const int np = T * (c.top_k + 1);
        if (qe_launch_bucket(sc.idx, T, c.E, c.top_k, T, 1, 1, 1, qe_group_tokens(), &sc.b, s) ||
            qe_launch_tc_prep(&m->ex, x, T, &sc.tcb, s))
            return -1;
        prof_mark(dev, s);
        if (qe_launch_group_gateup(&m->ex, &sc.tcb, T, &sc.b, sms, sc.h3, I, s)) return -1;
        prof_mark(dev, s);   /* the down stage includes the split of h3 */
        if (qe_launch_split_rows(c.bits, sc.h3, I, np, sc.tcb.h3s, sc.tcb.h3sum, sc.tcb.h3inv, s) ||
            qe_launch_group_down(&m->ex, &sc.tcb, np, &sc.b, sms, sc.ybuf, s))
            return -1;
        prof_mark(dev, s);
        if (qe_launch_combine(sc.ybuf, sc.score, sc.logits, c.E + 1, T, c.E, c.top_k, c.hidden, out, s)) return -1;
        prof_mark(dev, s);
        g_launches += 6;
        return 0;
    }
    const bool use_tc = m->tc && (m->path == 2 || (m->path == 0 && T >= kTcMinTokens));
    if (use_tc) {
        const int R = qe_tc_bm(), NB = m->tile ? m->tile : qe_tc_tokens_per_tile(T, c.top_k, c.E);
        const int tiles_gu = (c.inter + R - 1) / R, tiles_sh = (c.sh_inter + R - 1) / R,
                  tiles_dn = (c.hidden + R - 1) / R;
        if (qe_launch_bucket(sc.idx, T, c.E, c.top_k, T, tiles_gu, tiles_sh, tiles_dn, NB, &sc.b, s) ||
            qe_launch_tc_prep(&m->ex, x, T, &sc.tcb, s))
            return -1;
        prof_mark(dev, s);   /* the bucket stage includes the activation split, so gate/up times its kernel alone */
        if (qe_launch_tc_gateup(&m->ex, m->maps_gu, x, &sc.b, T, NB, &sc.tcb, sms, s)) return -1;
        prof_mark(dev, s);
        if (qe_launch_tc_down(&m->ex, m->maps_dn, &sc.b, T, NB, &sc.tcb, sc.ybuf, sms, s)) return -1;
        prof_mark(dev, s);
        if (qe_launch_combine(sc.ybuf, sc.score, sc.logits, c.E + 1, T, c.E, c.top_k, c.hidden, out, s)) return -1;
        prof_mark(dev, s);
        g_launches += 5;
        return 0;
    }
    const int R = qe_expert_rows_per_cta(T);
    const int tiles_gu = (c.inter + R - 1) / R, tiles_sh = (c.sh_inter + R - 1) / R, tiles_dn = (c.hidden + R - 1) / R;
    const int chunk = T < 8 ? T : 8;
    if (qe_launch_bucket(sc.idx, T, c.E, c.top_k, T, tiles_gu, tiles_sh, tiles_dn, chunk, &sc.b, s)) return -1;
    prof_mark(dev, s);
    /* grid: enough CTAs for every item in the common case, grid-stride beyond */
    const long long slots = std::min<long long>((long long)c.E, (long long)T * c.top_k) + 1;
    const long long chunks = ((long long)T * (c.top_k + 1) + chunk - 1) / chunk + slots;
    const int tmax = std::max(tiles_gu, tiles_sh);
    const int grid_gu = (int)std::min<long long>(chunks * tmax, 16LL * sms);
    const int grid_dn = (int)std::min<long long>(chunks * tiles_dn, 16LL * sms);
    if (qe_launch_gateup(&m->ex, x, &sc.b, T, sc.h3, I, grid_gu, s)) return -1;
    prof_mark(dev, s);
    if (qe_launch_down(&m->ex, sc.h3, I, &sc.b, T, sc.ybuf, grid_dn, s)) return -1;
    prof_mark(dev, s);
    if (qe_launch_combine(sc.ybuf, sc.score, sc.logits, c.E + 1, T, c.E, c.top_k, c.hidden, out, s)) return -1;
    prof_mark(dev, s);
    g_launches += 4;
    return 0;
}

/* ------------------------------------------------------------------ expert parallelism */

/* gate[t] = the shared-expert gate logit of token t (router column E). */
__global__ void ep_gate_kernel(const float *__restrict__ logits, int T, int E, float *__restrict__ gate) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < T) gate[t] = logits[(size_t)t * (E + 1) + E];
}

/* meta[T][2k]: the routing result per token, global expert ids then the scores' bits */
__global__ void ep_meta_kernel(const int32_t *__restrict__ idx, const float *__restrict__ score, int T, int k,
                               int32_t *__restrict__ meta) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * k) return;
    const int t = i / k, j = i % k;
    meta[(size_t)t * 2 * k + j] = idx[i];
    meta[(size_t)t * 2 * k + k + j] = __float_as_int(score[i]);
}

/* The expert placement on the device: per expert e, place[e*W] = its local slot on this rank (-1: not held),
 * place[e*W + 1] = replica count n, place[e*W + 2 ..] = the n holding ranks ascending (W = 2 + G). */
struct EpPlace {
    const int32_t *t;
    int W;
};

EpPlace place_of(const QeMoe *m) { return {m->place, 2 + m->cfg.ep_size}; }

/* The rank serving expert e for the token in row t of source rank src: replica (t + src) mod n. */
__device__ __forceinline__ int ep_dest(EpPlace p, int e, int t, int src) {
    const int32_t *te = p.t + (size_t)e * p.W;
    const int n = te[1];
    return te[2 + (n > 1 ? (t + src) % n : 0)];
}

/* meta -> local slot ids (-1 = not this rank's) and scores. Ids tagged QE_EP_ROUTED were routed here by the
 * sender; untagged ids (the replicated step's own meta, row = token) count where replica (row, src 0) is
 * this rank. */
__global__ void ep_local_kernel(const int32_t *__restrict__ meta, int n, int k, int self, EpPlace pl,
                                int32_t *__restrict__ idx, float *__restrict__ score) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * k) return;
    const int t = i / k, j = i % k;
    const int e = meta[(size_t)t * 2 * k + j];
    int s = -1;
    if (e >= 0) {
        const int g = e & ~QE_EP_ROUTED;
        if (e & QE_EP_ROUTED) s = pl.t[(size_t)g * pl.W];
        else if (ep_dest(pl, g, t, 0) == self) s = pl.t[(size_t)g * pl.W];
    }
    idx[i] = s;
    score[i] = __int_as_float(meta[(size_t)t * 2 * k + k + j]);
}

/* Slot j's id in the slot list sent to rank d: tagged if routed to d, else -1. */
__device__ __forceinline__ int32_t ep_sent_id(EpPlace pl, int32_t e, int t, int src, int d) {
    return e >= 0 && ep_dest(pl, e, t, src) == d ? (e | QE_EP_ROUTED) : -1;
}

/* One block per destination rank d: home[d][t] = the row of token t in block d (the tokens with at least one
 * slot routed to d, in token order) or -1, counts[d] = rows in block d. */
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t *__restrict__ meta, int T, int k, int src,
                                                       EpPlace pl, int32_t *__restrict__ home,
                                                       int32_t *__restrict__ counts) {
    const int d = blockIdx.x;
    __shared__ int wsum[32];
    __shared__ int base_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) base_s = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += 1024) {
        const int t = t0 + tid;
        int f = 0;
        if (t < T)
            for (int j = 0; j < k; j++) {
                const int e = meta[(size_t)t * 2 * k + j];
                f |= (e >= 0 && ep_dest(pl, e, t, src) == d) ? 1 : 0;
            }
        int incl = f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(QE_FULL, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int w = wsum[lane];
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(QE_FULL, wi, o);
                if (lane >= o) wi += v;
            }
            wsum[lane] = wi - w;
        }
        __syncthreads();
        const int base = base_s;
        if (t < T) home[(size_t)d * T + t] = f ? base + wsum[warp] + incl - f : -1;
        __syncthreads();
        if (tid == 1023) base_s = base + wsum[31] + incl;
        __syncthreads();
    }
    if (tid == 0) counts[d] = base_s;
}

/* Warp (d, t): token t's row and slot list (ids as ep_sent_id) to its row of block d; row t of block d, when at
 * or past counts[d], becomes padding (expert ids -1, scores 0). H % 4 == 0, 16-byte aligned rows. */
__global__ void ep_scatter_kernel(const float *__restrict__ x, const int32_t *__restrict__ meta, int T, int H, int k,
                                  int G, int self, EpPlace pl, const int32_t *__restrict__ home,
                                  const int32_t *__restrict__ counts, float *__restrict__ send_x,
                                  int32_t *__restrict__ send_meta) {
    const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (long long)G * T) return;
    const int d = (int)(w / T), t = (int)(w % T);
    const int pos = home[(size_t)d * T + t];
    if (pos >= 0) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * H);
        float4 *dst = reinterpret_cast<float4 *>(send_x + ((size_t)d * T + pos) * H);
        for (int c = lane; c < H / 4; c += 32) dst[c] = src[c];
        for (int c = lane; c < 2 * k; c += 32) {
            const int32_t v = meta[(size_t)t * 2 * k + c];
            send_meta[((size_t)d * T + pos) * 2 * k + c] = c < k ? ep_sent_id(pl, v, t, self, d) : v;
        }
    }
    if (t >= counts[d])
        for (int c = lane; c < 2 * k; c += 32) send_meta[((size_t)d * T + t) * 2 * k + c] = c < k ? -1 : 0;
}

/* out[t] = (sum over ranks d ascending of part[d][home[d][t]], skipping -1) + shared[t]; home NULL: part[d][t] */
__global__ void ep_combine_kernel(const float *__restrict__ part, const int32_t *__restrict__ home,
                                  const float *__restrict__ shared, int T, int G, int H, float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T * H) return;
    const int t = (int)(i / H), c = (int)(i % H);
    float o = 0.0f;
    for (int d = 0; d < G; d++) {
        const int pos = home ? home[(size_t)d * T + t] : t;
        if (pos >= 0) o = __fadd_rn(o, part[((size_t)d * T + pos) * H + c]);
    }
    out[i] = __fadd_rn(o, shared[i]);
}

/* Where the expert stage's partial rows go when they are written into the home ranks' return buffers. */
struct EpScatter {
    float *const *base;   /* device [G]: every rank's return buffer */
    int row0, Tblk, self;
};

/* The rank's own tokens appended to the received rows (rows sh0 .. sh0 + sh_n - 1 of the pass, no routed slot):
 * the shared expert runs on them in the same launches, and sigmoid(gate[i]) * y_shared goes to sh_out[i]. */
struct EpFold {
    int sh0, sh_n;
    const float *gate;
    float *sh_out;
};

/* The expert stages for n rows whose local slot ids and scores are in sc.idx / sc.score (and, for the shared
 * expert, whose gate logits are in sc.logits): bucket, gate/up + SwiGLU, down, then the selective combine
 * into out[n][hidden], or (scatter) into the home ranks' return buffers. q is the rows the path choice counts:
 * the routed rows a rank receives (G x T in a token-sharded step), also for the shared-expert pass of T rows and
 * for a folded pass, so that the shared expert takes the same kernels either way. */
int run_experts(QeMoe *m, const float *x, float *out, int n, int q, Scratch &sc, int sms, bool routed, bool shared,
                cudaStream_t s, const EpScatter *scatter = nullptr, const EpFold *fold = nullptr) {
    const QeMoeConfig &c = m->cfg;
    const int El = m->E_loc, k = c.top_k;
    const int I = c.inter > c.sh_inter ? c.inter : c.sh_inter;
    const int sh_tokens = fold ? fold->sh_n : shared ? n : 0, sh0 = fold ? fold->sh0 : 0;
    const bool use_group = group_path(m, q);
    const bool use_tc = !use_group && m->tc && (m->path == 2 || (m->path == 0 && n >= kTcMinTokens));
    if (use_group) {
        const int np = n * (k + 1);
        if (qe_launch_bucket(sc.idx, n, El, k, sh_tokens, 1, 1, 1, qe_group_tokens(), &sc.b, s, sh0) ||
            qe_launch_tc_prep(&m->ex, x, n, &sc.tcb, s) ||
            qe_launch_group_gateup(&m->ex, &sc.tcb, n, &sc.b, sms, sc.h3, I, s) ||
            qe_launch_split_rows(c.bits, sc.h3, I, np, sc.tcb.h3s, sc.tcb.h3sum, sc.tcb.h3inv, s) ||
            qe_launch_group_down(&m->ex, &sc.tcb, np, &sc.b, sms, sc.ybuf, s))
            return -1;
        g_launches += 5;
    } else if (use_tc) {
        const int R = qe_tc_bm(), NB = m->tile ? m->tile : qe_tc_tokens_per_tile(n, c.top_k, c.E);
        const int tiles_gu = (c.inter + R - 1) / R, tiles_sh = (c.sh_inter + R - 1) / R,
                  tiles_dn = (c.hidden + R - 1) / R;
        if (qe_launch_bucket(sc.idx, n, El, k, sh_tokens, tiles_gu, tiles_sh, tiles_dn, NB, &sc.b, s, sh0) ||
            qe_launch_tc_prep(&m->ex, x, n, &sc.tcb, s) ||
            qe_launch_tc_gateup(&m->ex, m->maps_gu, x, &sc.b, n, NB, &sc.tcb, sms, s) ||
            qe_launch_tc_down(&m->ex, m->maps_dn, &sc.b, n, NB, &sc.tcb, sc.ybuf, sms, s))
            return -1;
        g_launches += 4;
    } else {
        const int R = qe_expert_rows_per_cta(n);
        const int tiles_gu = (c.inter + R - 1) / R, tiles_sh = (c.sh_inter + R - 1) / R,
                  tiles_dn = (c.hidden + R - 1) / R;
        const int chunk = n < 8 ? n : 8;
        const long long slots = std::min<long long>((long long)El, (long long)n * k) + 1;
        const long long chunks = ((long long)n * (k + 1) + chunk - 1) / chunk + slots;
        const int tmax = std::max(tiles_gu, tiles_sh);
        const int grid_gu = (int)std::min<long long>(chunks * tmax, 16LL * sms);
        const int grid_dn = (int)std::min<long long>(chunks * tiles_dn, 16LL * sms);
        if (qe_launch_bucket(sc.idx, n, El, k, sh_tokens, tiles_gu, tiles_sh, tiles_dn, chunk, &sc.b, s, sh0) ||
            qe_launch_gateup(&m->ex, x, &sc.b, n, sc.h3, I, grid_gu, s) ||
            qe_launch_down(&m->ex, sc.h3, I, &sc.b, n, sc.ybuf, grid_dn, s))
            return -1;
        g_launches += 3;
    }
    if (fold) {
        /* received rows [0, sh0): partial sums into the home ranks; own rows: the gated shared expert */
        const size_t H = c.hidden;
        if (sh0 > 0 && qe_launch_combine_sel_scatter(sc.ybuf, sc.idx, sc.score, sh0, k, c.hidden, scatter->base,
                                                     scatter->row0, scatter->Tblk, scatter->self, s))
            return -1;
        if (fold->sh_n > 0 &&
            qe_launch_combine_sel(sc.ybuf + (size_t)sh0 * (k + 1) * H, sc.idx + (size_t)sh0 * k,
                                  sc.score + (size_t)sh0 * k, fold->gate, 1, fold->sh_n, 0, k, c.hidden, 0, 1,
                                  fold->sh_out, s))
            return -1;
        g_launches += (sh0 > 0) + (fold->sh_n > 0);
        return 0;
    }
    if (scatter) {
        if (qe_launch_combine_sel_scatter(sc.ybuf, sc.idx, sc.score, n, k, c.hidden, scatter->base, scatter->row0,
                                          scatter->Tblk, scatter->self, s))
            return -1;
    } else if (qe_launch_combine_sel(sc.ybuf, sc.idx, sc.score, sc.logits, c.E + 1, n, c.E, k, c.hidden,
                                     routed ? 1 : 0, shared ? 1 : 0, out, s)) {
        return -1;
    }
    g_launches += 1;
    return 0;
}

/* Warp (d, t), peer-memory dispatch: token t's row and slot list go straight into rank d's receive buffers,
 * block `self`, row home[d][t]; row t of that block at or past counts[d] becomes padding. */
__global__ void ep_scatter_p2p_kernel(const float *__restrict__ x, const int32_t *__restrict__ meta, int T, int H,
                                      int k, int G, int self, EpPlace pl, const int32_t *__restrict__ home,
                                      const int32_t *__restrict__ counts, float *const *__restrict__ recv_x,
                                      int32_t *const *__restrict__ recv_meta) {
    const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (long long)G * T) return;
    const int d = (int)(w / T), t = (int)(w % T);
    const int pos = home[(size_t)d * T + t];
    if (pos >= 0) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * H);
        float4 *dst = reinterpret_cast<float4 *>(recv_x[d] + ((size_t)self * T + pos) * H);
        for (int c = lane; c < H / 4; c += 32) dst[c] = src[c];
        int32_t *dm = recv_meta[d] + ((size_t)self * T + pos) * 2 * k;
        for (int c = lane; c < 2 * k; c += 32) {
            const int32_t v = meta[(size_t)t * 2 * k + c];
            dm[c] = c < k ? ep_sent_id(pl, v, t, self, d) : v;
        }
    }
    if (t >= counts[d]) {
        int32_t *dm = recv_meta[d] + ((size_t)self * T + t) * 2 * k;
        for (int c = lane; c < 2 * k; c += 32) dm[c] = c < k ? -1 : 0;
    }
    __threadfence_system();
}

void trace_route(const QeMoe *m, const int32_t *idx, int T) {
    /* QE_TRACE=<file>: append int32 layer, idx[top_k] per token (engine/src/moe_layer.c:57-64) */
    static FILE *f;
    static int checked;
    if (!checked) {
        const char *p = getenv("QE_TRACE");
        f = p ? fopen(p, "ab") : nullptr;
        checked = 1;
    }
    if (!f) return;
    const int32_t layer = m->cfg.layer;
    for (int t = 0; t < T; t++) {
        fwrite(&layer, 4, 1, f);
        fwrite(idx + (size_t)t * m->cfg.top_k, 4, (size_t)m->cfg.top_k, f);
    }
    fflush(f);
}

}  // namespace

extern "C" {

int qe_moe_forward_device(QeMoe *m, int T, const float *x, float *out, void *stream) {
    if (!m || !x || !out || T < 1) QE_FAIL("forward: bad arguments");
    if (m->cfg.ep_size > 1) QE_FAIL("forward: this handle holds %d of the %d experts only: use the qe_moe_ep_* calls",
                                    m->E_loc, m->cfg.E);
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const int P = std::min(T, m->cfg.max_tokens);
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    for (int t0 = 0; t0 < T; t0 += P) {
        const int n = std::min(P, T - t0);
        const size_t o = (size_t)t0 * m->cfg.hidden;
        if (run_pass(m, x + o, out + o, n, sc, d->sms, s)) return -1;
    }
    return 0;
}

struct QeMoeGraph {
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    void *ws;                      /* the graph's own scratch (the shared workspace may be reallocated) */
    int device;
    unsigned long long launches;   /* kernels in one replay */
};

}  // extern "C"

namespace {
/* qe_moe_forward_device on a given scratch workspace */
int forward_ws(QeMoe *m, int T, const float *x, float *out, char *ws, int sms, cudaStream_t s) {
    const int P = std::min(T, m->cfg.max_tokens);
    Scratch sc;
    scratch_layout(m->cfg, P, ws, &sc);
    for (int t0 = 0; t0 < T; t0 += P) {
        const int n = std::min(P, T - t0);
        const size_t o = (size_t)t0 * m->cfg.hidden;
        if (run_pass(m, x + o, out + o, n, sc, sms, s)) return -1;
    }
    return 0;
}
}  // namespace

extern "C" {

QeMoeGraph *qe_moe_graph_create(QeMoe *m, int T, const float *x, float *out) {
    if (!m || !x || !out || T < 1 || m->cfg.ep_size > 1) {
        fprintf(stderr, "qengine_b200: graph_create: bad arguments\n");
        return nullptr;
    }
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return nullptr;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    QeMoeGraph *g = (QeMoeGraph *)calloc(1, sizeof(QeMoeGraph));
    bool ok = g != nullptr;
    const size_t wsb = scratch_layout(m->cfg, std::min(T, m->cfg.max_tokens), nullptr, nullptr);
    ok = ok && cudaMalloc(&g->ws, wsb) == cudaSuccess;
    /* one eager forward first: kernel attributes set (that may not happen during capture) */
    ok = ok && forward_ws(m, T, x, out, (char *)g->ws, d->sms, s) == 0 && cudaStreamSynchronize(s) == cudaSuccess;
    const unsigned long long l0 = g_launches.load();
    ok = ok && cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
        const int rc = forward_ws(m, T, x, out, (char *)g->ws, d->sms, s);
        cudaGraph_t graph = nullptr;
        const bool ended = cudaStreamEndCapture(s, &graph) == cudaSuccess;
        ok = rc == 0 && ended;
        if (ok) {
            g->graph = graph;
            ok = cudaGraphInstantiate(&g->exec, graph, 0) == cudaSuccess;
        } else if (graph) {
            cudaGraphDestroy(graph);
        }
    }
    cudaStreamDestroy(s);
    if (!ok) {
        fprintf(stderr, "qengine_b200: graph_create: capture failed\n");
        if (g) {
            if (g->exec) cudaGraphExecDestroy(g->exec);
            if (g->graph) cudaGraphDestroy(g->graph);
            if (g->ws) cudaFree(g->ws);
            free(g);
        }
        return nullptr;
    }
    g->device = m->device;
    g->launches = g_launches.load() - l0;
    g_captures += 1;
    return g;
}

int qe_moe_graph_launch(QeMoeGraph *g, void *stream) {
    if (!g) QE_FAIL("graph_launch: null graph");
    QE_CHECK(cudaSetDevice(g->device));
    QE_CHECK(cudaGraphLaunch(g->exec, (cudaStream_t)stream));
    g_launches += g->launches;
    return 0;
}

void qe_moe_graph_free(QeMoeGraph *g) {
    if (!g) return;
    cudaSetDevice(g->device);
    cudaGraphExecDestroy(g->exec);
    cudaGraphDestroy(g->graph);
    cudaFree(g->ws);
    free(g);
}

/* Pipelined forward with host buffers. Call i uses staging slot i % 2: its x copy (copy-in stream) waits until
 * the forward of call i - 2 has read the slot, its forward (the device stream) waits for the copy and for call
 * i - 2's out copy, and its out copy (copy-out stream) waits for the forward. So the copies of neighbouring
 * calls run under each other's kernels; every call computes what qe_moe_forward does. */
int qe_moe_forward_async(QeMoe *m, int T, const float *x, float *out) {
    if (!m || !x || !out || T < 1) QE_FAIL("forward_async: bad arguments");
    if (m->cfg.ep_size > 1) QE_FAIL("forward_async: this handle holds %d of the %d experts only: use the qe_moe_ep_* calls",
                                    m->E_loc, m->cfg.E);
    if (T > m->cfg.max_tokens) QE_FAIL("forward_async: T=%d above the handle's max_tokens %d", T, m->cfg.max_tokens);
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = d->stream;
    if (ensure_ws(d, scratch_layout(m->cfg, T, nullptr, nullptr))) return -1;
    if (!d->s_in) {
        QE_CHECK(cudaStreamCreateWithFlags(&d->s_in, cudaStreamNonBlocking));
        QE_CHECK(cudaStreamCreateWithFlags(&d->s_out, cudaStreamNonBlocking));
        for (int j = 0; j < 2; j++) {
            QE_CHECK(cudaEventCreateWithFlags(&d->ev_h2d[j], cudaEventDisableTiming));
            QE_CHECK(cudaEventCreateWithFlags(&d->ev_comp[j], cudaEventDisableTiming));
            QE_CHECK(cudaEventCreateWithFlags(&d->ev_d2h[j], cudaEventDisableTiming));
        }
    }
    const size_t nf = (size_t)T * m->cfg.hidden;
    if (d->stage_cap < nf) {
        QE_CHECK(cudaDeviceSynchronize());   /* no call in flight uses the old staging memory */
        if (d->stage) cudaFree(d->stage);
        d->stage = nullptr;
        d->stage_cap = 0;
        QE_CHECK(cudaMalloc((void **)&d->stage, sizeof(float) * 4 * nf));
        d->stage_cap = nf;
        d->slot_used[0] = d->slot_used[1] = false;
    }
    Scratch sc;
    scratch_layout(m->cfg, T, (char *)d->ws, &sc);
    const int j = (int)(d->async_n++ & 1);
    float *xd = d->stage + (size_t)(2 * j) * d->stage_cap, *od = xd + d->stage_cap;
    /* The forward is replayed from a CUDA graph captured for this handle, staging slot and T (no per-kernel launch
     * gaps). The graphs of BOTH slots are captured together, on the handle's first call with this T (or after the
     * staging buffers grew), with the device idle, since each capture runs an eager forward on the slot's
     * buffers; later calls with the same T never capture, whichever slot they get. */
    static const bool use_graph = !getenv("QE_ASYNC_GRAPH") || strcmp(getenv("QE_ASYNC_GRAPH"), "0") != 0;
    if (use_graph && !(m->agraph[j] && m->a_T[j] == T && m->a_x[j] == xd && m->a_o[j] == od)) {
        QE_CHECK(cudaDeviceSynchronize());
        for (int q = 0; q < 2; q++) {
            float *xq = d->stage + (size_t)(2 * q) * d->stage_cap, *oq = xq + d->stage_cap;
            if (m->agraph[q] && m->a_T[q] == T && m->a_x[q] == xq && m->a_o[q] == oq) continue;
            qe_moe_graph_free(m->agraph[q]);
            m->agraph[q] = qe_moe_graph_create(m, T, xq, oq);
            if (!m->agraph[q]) QE_FAIL("forward_async: graph capture failed");
            m->a_T[q] = T;
            m->a_x[q] = xq;
            m->a_o[q] = oq;
        }
    }
    if (d->slot_used[j]) QE_CHECK(cudaStreamWaitEvent(d->s_in, d->ev_comp[j], 0));
    QE_CHECK(cudaMemcpyAsync(xd, x, sizeof(float) * nf, cudaMemcpyHostToDevice, d->s_in));
    QE_CHECK(cudaEventRecord(d->ev_h2d[j], d->s_in));
    QE_CHECK(cudaStreamWaitEvent(s, d->ev_h2d[j], 0));
    if (d->slot_used[j]) QE_CHECK(cudaStreamWaitEvent(s, d->ev_d2h[j], 0));
    if (use_graph) {
        if (qe_moe_graph_launch(m->agraph[j], s)) return -1;
    } else if (run_pass(m, xd, od, T, sc, d->sms, s)) {
        return -1;
    }
    QE_CHECK(cudaEventRecord(d->ev_comp[j], s));
    QE_CHECK(cudaStreamWaitEvent(d->s_out, d->ev_comp[j], 0));
    QE_CHECK(cudaMemcpyAsync(out, od, sizeof(float) * nf, cudaMemcpyDeviceToHost, d->s_out));
    QE_CHECK(cudaEventRecord(d->ev_d2h[j], d->s_out));
    d->slot_used[j] = true;
    return 0;
}

int qe_moe_forward_wait(QeMoe *m) {
    if (!m) QE_FAIL("forward_wait: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    if (d->s_out) QE_CHECK(cudaStreamSynchronize(d->s_out));
    QE_CHECK(cudaStreamSynchronize(d->stream));
    return 0;
}

/* For a caller that runs qe_moe_forward_device inside its own step (the GPU trunk of the whole-model API): what
 * qe_moe_forward does after a decode batch of T tokens -- the selected experts' bytes added to the read statistics
 * (T * top_k experts, as qe_moe_forward counts a decode batch) and, when QE_TRACE is set and a stream is given, the
 * step's routing appended to the trace file (read back from the workspace the forward used -- ws, or the device's
 * shared one when null -- after the stream's work so far; T within one pass). */
int qe_moe_note_device_forward(QeMoe *m, int T, void *ws, void *stream) {
    if (!m || T < 1) return -1;
    g_bytes_read += (unsigned long long)T * m->cfg.top_k * (unsigned long long)m->expert_bytes;
    if (!stream || !getenv("QE_TRACE") || T > m->cfg.max_tokens) return 0;   /* no stream: statistics only */
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    Scratch sc;
    scratch_layout(m->cfg, std::min(T, m->cfg.max_tokens), ws ? (char *)ws : (char *)d->ws, &sc);
    std::vector<int32_t> idx((size_t)T * m->cfg.top_k);
    cudaStream_t s = (cudaStream_t)stream;
    QE_CHECK(cudaMemcpyAsync(idx.data(), sc.idx, 4 * idx.size(), cudaMemcpyDeviceToHost, s));
    QE_CHECK(cudaStreamSynchronize(s));
    trace_route(m, idx.data(), T);
    return 0;
}

/* qe_moe_forward_device on a workspace of the caller's (qe_moe_ws_bytes(m, T) bytes of device memory): for a
 * caller that captures its own step in a CUDA graph, whose pointers must not move when the device's shared
 * workspace grows for another call. */
size_t qe_moe_ws_bytes(const QeMoe *m, int T) {
    return m && T > 0 ? scratch_layout(m->cfg, std::min(T, m->cfg.max_tokens), nullptr, nullptr) : 0;
}
int qe_moe_forward_device_ws(QeMoe *m, int T, const float *x, float *out, void *ws, void *stream) {
    if (!m || !x || !out || !ws || T < 1 || m->cfg.ep_size > 1) QE_FAIL("forward_ws: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    return forward_ws(m, T, x, out, (char *)ws, d->sms, (cudaStream_t)stream);
}

int qe_moe_forward(QeMoe *m, int T, const float *x, float *out) {
    if (!m || !x || !out || T < 1) QE_FAIL("forward: bad arguments");
    if (m->cfg.ep_size > 1) QE_FAIL("forward: this handle holds %d of the %d experts only: use the qe_moe_ep_* calls",
                                    m->E_loc, m->cfg.E);
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = d->stream;
    const int P = std::min(T, m->cfg.max_tokens);
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    const size_t H = m->cfg.hidden;
    const bool tracing = getenv("QE_TRACE") != nullptr;
    std::vector<int32_t> idx_host;
    unsigned long long experts_touched = 0;
    QE_CHECK(cudaEventRecord(d->ev0, s));
    for (int t0 = 0; t0 < T; t0 += P) {
        const int n = std::min(P, T - t0);
        QE_CHECK(cudaMemcpyAsync(sc.x, x + (size_t)t0 * H, sizeof(float) * n * H, cudaMemcpyHostToDevice, s));
        if (run_pass(m, sc.x, sc.out, n, sc, d->sms, s)) return -1;
        QE_CHECK(cudaMemcpyAsync(out + (size_t)t0 * H, sc.out, sizeof(float) * n * H, cudaMemcpyDeviceToHost, s));
        /* experts read by this pass: the active buckets (bucketed paths), or every selected slot plus the
         * shared expert (decode path, no buckets: an upper bound when tokens share experts) */
        const bool decode = m->decode && (m->path == 3 || (m->path == 0 && n <= kDecodeMaxTokens));
        int32_t na = n * m->cfg.top_k + 1;
        if (!decode) QE_CHECK(cudaMemcpyAsync(&na, sc.b.n_active, 4, cudaMemcpyDeviceToHost, s));
        if (tracing) {
            idx_host.resize((size_t)n * m->cfg.top_k);
            QE_CHECK(cudaMemcpyAsync(idx_host.data(), sc.idx, 4 * idx_host.size(), cudaMemcpyDeviceToHost, s));
        }
        QE_CHECK(cudaStreamSynchronize(s));
        experts_touched += (unsigned long long)(na > 0 ? na - 1 : 0);
        if (tracing) trace_route(m, idx_host.data(), n);
    }
    QE_CHECK(cudaEventRecord(d->ev1, s));
    QE_CHECK(cudaEventSynchronize(d->ev1));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, d->ev0, d->ev1);
    g_gpu_seconds += ms * 1e-3;
    g_bytes_read += experts_touched * (unsigned long long)m->expert_bytes;
    return 0;
}

int qe_moe_route(QeMoe *m, int T, const float *x, int32_t *idx, float *score) {
    if (!m || !x || !idx || !score || T < 1) QE_FAIL("route: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = d->stream;
    const int P = std::min(T, m->cfg.max_tokens);
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    const size_t H = m->cfg.hidden, k = m->cfg.top_k;
    for (int t0 = 0; t0 < T; t0 += P) {
        const int n = std::min(P, T - t0);
        QE_CHECK(cudaMemcpyAsync(sc.x, x + (size_t)t0 * H, sizeof(float) * n * H, cudaMemcpyHostToDevice, s));
        if (run_route(m, sc.x, n, sc, s)) return -1;
        QE_CHECK(cudaMemcpyAsync(idx + (size_t)t0 * k, sc.idx, 4 * n * k, cudaMemcpyDeviceToHost, s));
        QE_CHECK(cudaMemcpyAsync(score + (size_t)t0 * k, sc.score, 4 * n * k, cudaMemcpyDeviceToHost, s));
        QE_CHECK(cudaStreamSynchronize(s));
    }
    return 0;
}

int qe_moe_ep_size(const QeMoe *m) { return m ? m->cfg.ep_size : -1; }

int qe_moe_ep_experts(const QeMoe *m, int32_t *ids) {
    if (!m) return -1;
    if (ids) memcpy(ids, m->held, sizeof(int32_t) * m->E_loc);
    return m->E_loc;
}

int qe_moe_ep_route_device(QeMoe *m, int T, const float *x, int32_t *meta, float *shared, void *stream) {
    if (!m || !x || !meta || !shared || T < 1) QE_FAIL("ep_route: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const int P = std::min(T, m->cfg.max_tokens), k = m->cfg.top_k;
    const size_t H = m->cfg.hidden;
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    for (int t0 = 0; t0 < T; t0 += P) {
        const int n = std::min(P, T - t0);
        if (run_route(m, x + (size_t)t0 * H, n, sc, s)) return -1;
        ep_meta_kernel<<<(n * k + 255) / 256, 256, 0, s>>>(sc.idx, sc.score, n, k, meta + (size_t)t0 * 2 * k);
        QE_CHECK(cudaGetLastError());
        QE_CHECK(cudaMemsetAsync(sc.idx, 0xff, sizeof(int32_t) * (size_t)n * k, s));   /* shared expert only */
        if (run_experts(m, x + (size_t)t0 * H, shared + (size_t)t0 * H, n, n * m->cfg.ep_size, sc, d->sms, false, true,
                        s))
            return -1;
        g_launches += 1;   /* ep_meta_kernel */
    }
    return 0;
}

int qe_moe_ep_pack_device(QeMoe *m, int T, const float *x, const int32_t *meta, float *send_x, int32_t *send_meta,
                          int32_t *home, int32_t *counts, void *stream) {
    if (!m || !x || !meta || !send_x || !send_meta || !home || !counts || T < 1) QE_FAIL("ep_pack: bad arguments");
    const int H = m->cfg.hidden, k = m->cfg.top_k, G = m->cfg.ep_size;
    if (H % 4 || ((uintptr_t)x | (uintptr_t)send_x) % 16) QE_FAIL("ep_pack: x and send_x must be 16-byte aligned");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    ep_plan_kernel<<<G, 1024, 0, s>>>(meta, T, k, m->cfg.ep_rank, place_of(m), home, counts);
    QE_CHECK(cudaGetLastError());
    const long long threads = (long long)G * T * 32;
    ep_scatter_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, meta, T, H, k, G, m->cfg.ep_rank,
                                                                       place_of(m), home, counts, send_x, send_meta);
    QE_CHECK(cudaGetLastError());
    g_launches += 2;
    return 0;
}

int qe_moe_ep_experts_device(QeMoe *m, int n, const float *x, const int32_t *meta, float *partial, void *stream) {
    if (!m || !x || !meta || !partial || n < 1) QE_FAIL("ep_experts: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const int P = std::min(n, m->cfg.max_tokens), k = m->cfg.top_k;
    const size_t H = m->cfg.hidden;
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    for (int r0 = 0; r0 < n; r0 += P) {
        const int cnt = std::min(P, n - r0);
        ep_local_kernel<<<(cnt * k + 255) / 256, 256, 0, s>>>(meta + (size_t)r0 * 2 * k, cnt, k, m->cfg.ep_rank,
                                                             place_of(m), sc.idx, sc.score);
        QE_CHECK(cudaGetLastError());
        if (run_experts(m, x + (size_t)r0 * H, partial + (size_t)r0 * H, cnt, cnt, sc, d->sms, true, false, s)) return -1;
        g_launches += 1;
    }
    return 0;
}

int qe_moe_ep_combine_device(QeMoe *m, int T, const float *part, const int32_t *home, const float *shared, float *out,
                             void *stream) {
    if (!m || !part || !shared || !out || T < 1) QE_FAIL("ep_combine: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    const long long n = (long long)T * m->cfg.hidden;
    ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(part, home, shared, T,
                                                                                     m->cfg.ep_size,
                                                                                     m->cfg.hidden, out);
    QE_CHECK(cudaGetLastError());
    g_launches += 1;
    return 0;
}

/* ---- expert-parallel exchange through peer memory (CUDA IPC mappings of every rank's buffers) ---- */

}  // extern "C"

struct QeEpXchg {
    QeMoe *m;
    int G, self, Tmax, H, k;
    char *mine;                      /* this rank's buffers: recv_x [G+1][Tmax][H] (block G: its own rows, written by
                                      * qe_moe_ep_route_p2p), recv_meta [G][Tmax][2k], back [G][Tmax][H],
                                      * gate [Tmax] (own tokens' shared-expert gate logits), shared [Tmax][H],
                                      * flags [1 + G] u32 (qe_ep_xchg_barrier: epoch counter, then one slot per
                                      * rank written by that rank) */
    size_t off_meta, off_back, off_gate, off_shared, off_flags, bytes;
    int fold_T;                      /* T of a step routed by qe_moe_ep_route_p2p (shared expert in the expert
                                      * stage), until its combine; else 0 */
    char *base[64];                  /* every rank's allocation as mapped here (own = mine)                      */
    bool opened[64];
    void **dptr;                     /* device arrays: recv_x[G], recv_meta[G], back[G]                          */
    int T;                           /* tokens per rank of the current step                                     */
    unsigned long long wait_ns;      /* bound of each wait in qe_ep_xchg_barrier (qe_ep_xchg_set_timeout_ms)    */
};

namespace {
__device__ int g_ep_error;   /* first exchange-barrier timeout, read by qe_device_error() */

__device__ __forceinline__ uint64_t ep_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* Barrier across the ranks of the peer-memory exchange, one warp. The epoch is this rank's counter flags[self][0]
 * plus one (every rank calls the barrier the same number of times, so the counters agree, also when the call
 * is replayed from a CUDA graph). Lane r publishes the epoch into rank r's slot for this rank, after a system
 * fence that orders this stream's earlier stores into the peers' buffers; then lane r waits, for at most
 * wait_ns, until rank r's slot in this rank's flags reaches the epoch (a slot only grows). On timeout it
 * records g_ep_error and returns. */
__global__ void ep_barrier_kernel(unsigned *const *__restrict__ flags, int self, int G, unsigned long long wait_ns) {
    const int lane = threadIdx.x;
    unsigned *mine = flags[self];
    const unsigned epoch = *(volatile unsigned *)mine + 1u;
    __syncwarp();
    __threadfence_system();
    if (lane < G) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags[lane] + 1 + self), "r"(epoch) : "memory");
    if (lane < G) {
        const uint64_t t0 = ep_timer_ns();
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + 1 + lane) : "memory");
            if ((int)(v - epoch) >= 0) break;
            if (ep_timer_ns() - t0 > wait_ns) {
                atomicCAS(&g_ep_error, 0, 1);
                break;
            }
        }
    }
    __syncwarp();
    if (lane == 0) *(volatile unsigned *)mine = epoch;
    __threadfence_system();
}

/* The three buffers are laid out for the step's T (blocks of T rows), within the Tmax capacity. */
void xchg_tables(QeEpXchg *x, int T, void **host) {
    for (int r = 0; r < x->G; r++) {
        char *b = x->base[r];
        host[r] = b;
        host[x->G + r] = b + x->off_meta;
        host[2 * x->G + r] = b + x->off_back;
        host[3 * x->G + r] = b + x->off_flags;
    }
    (void)T;
}
}  // namespace

extern "C" {

QeEpXchg *qe_ep_xchg_create(QeMoe *m, int T_max, void *handle) {
    if (!m || T_max < 1 || !handle) {
        fprintf(stderr, "qengine_b200: ep_xchg_create: bad arguments\n");
        return nullptr;
    }
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return nullptr;
    QeEpXchg *x = (QeEpXchg *)calloc(1, sizeof(QeEpXchg));
    if (!x) return nullptr;
    x->m = m;
    x->G = m->cfg.ep_size;
    x->self = m->cfg.ep_rank;
    x->Tmax = T_max;
    x->H = m->cfg.hidden;
    x->k = m->cfg.top_k;
    const size_t rows = (size_t)x->G * T_max;
    x->off_meta = align256((rows + T_max) * x->H * 4);
    x->off_back = x->off_meta + align256(rows * 2 * x->k * 4);
    x->off_gate = x->off_back + align256(rows * x->H * 4);
    x->off_shared = x->off_gate + align256((size_t)T_max * 4);
    x->off_flags = x->off_shared + align256((size_t)T_max * x->H * 4);
    x->bytes = x->off_flags + align256(sizeof(unsigned) * (1 + (size_t)x->G));
    if (cudaMalloc((void **)&x->mine, x->bytes) != cudaSuccess ||
        cudaMalloc((void **)&x->dptr, sizeof(void *) * 4 * x->G) != cudaSuccess ||
        cudaMemset(x->mine + x->off_flags, 0, sizeof(unsigned) * (1 + (size_t)x->G)) != cudaSuccess ||
        cudaIpcGetMemHandle((cudaIpcMemHandle_t *)handle, x->mine) != cudaSuccess) {
        fprintf(stderr, "qengine_b200: ep_xchg_create: cannot allocate or export %zu bytes\n", x->bytes);
        if (x->mine) cudaFree(x->mine);
        if (x->dptr) cudaFree(x->dptr);
        free(x);
        return nullptr;
    }
    x->base[x->self] = x->mine;
    return x;
}

int qe_ep_xchg_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int qe_ep_xchg_connect(QeEpXchg *x, const void *handles) {
    if (!x || !handles) QE_FAIL("ep_xchg_connect: bad arguments");
    QE_CHECK(cudaSetDevice(x->m->device));
    for (int r = 0; r < x->G; r++) {
        if (r == x->self || x->opened[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const char *)handles + (size_t)r * sizeof(h), sizeof(h));
        void *p = nullptr;
        QE_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        x->base[r] = (char *)p;
        x->opened[r] = true;
    }
    void *host[4 * 64];
    xchg_tables(x, 0, host);
    QE_CHECK(cudaMemcpy(x->dptr, host, sizeof(void *) * 4 * x->G, cudaMemcpyHostToDevice));
    return 0;
}

int qe_ep_xchg_connect_local(QeEpXchg *const *all, int n) {
    /* ranks emulated in one process on one device: the buffers are plain device pointers */
    if (!all || n < 1) QE_FAIL("ep_xchg_connect_local: bad arguments");
    for (int i = 0; i < n; i++) {
        QeEpXchg *x = all[i];
        if (!x || x->G != n) QE_FAIL("ep_xchg_connect_local: %d contexts for ep_size %d", n, x ? x->G : -1);
        for (int r = 0; r < n; r++) x->base[r] = all[r]->mine;
        void *host[4 * 64];
        xchg_tables(x, 0, host);
        QE_CHECK(cudaSetDevice(x->m->device));
        QE_CHECK(cudaMemcpy(x->dptr, host, sizeof(void *) * 4 * x->G, cudaMemcpyHostToDevice));
    }
    return 0;
}

void qe_ep_xchg_free(QeEpXchg *x) {
    if (!x) return;
    cudaSetDevice(x->m->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < x->G; r++)
        if (x->opened[r]) cudaIpcCloseMemHandle(x->base[r]);
    cudaFree(x->dptr);
    cudaFree(x->mine);
    free(x);
}

int qe_ep_xchg_barrier(QeEpXchg *x, void *stream) {
    if (!x) QE_FAIL("ep_xchg_barrier: bad arguments");
    if (x->G > 32) QE_FAIL("ep_xchg_barrier: %d ranks (one warp serves at most 32)", x->G);
    QE_CHECK(cudaSetDevice(x->m->device));
    ep_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned *const *)(x->dptr + 3 * x->G), x->self, x->G,
                                                         x->wait_ns ? x->wait_ns : 2000000000ull);
    QE_CHECK(cudaGetLastError());
    g_launches += 1;
    return 0;
}

int qe_moe_ep_dispatch_p2p(QeMoe *m, QeEpXchg *xc, int T, const float *x, const int32_t *meta, int32_t *home,
                           int32_t *counts, void *stream) {
    if (!m || !xc || !x || !meta || !home || !counts || T < 1 || T > xc->Tmax) QE_FAIL("ep_dispatch_p2p: bad arguments");
    const int H = m->cfg.hidden, k = m->cfg.top_k, G = m->cfg.ep_size;
    if (H % 4 || (uintptr_t)x % 16) QE_FAIL("ep_dispatch_p2p: x must be 16-byte aligned");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    ep_plan_kernel<<<G, 1024, 0, s>>>(meta, T, k, m->cfg.ep_rank, place_of(m), home, counts);
    QE_CHECK(cudaGetLastError());
    const long long threads = (long long)G * T * 32;
    ep_scatter_p2p_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
        x, meta, T, H, k, G, m->cfg.ep_rank, place_of(m), home, counts, (float *const *)xc->dptr,
        (int32_t *const *)(xc->dptr + G));
    QE_CHECK(cudaGetLastError());
    xc->T = T;
    g_launches += 2;
    return 0;
}

int qe_moe_ep_route_p2p(QeMoe *m, QeEpXchg *xc, int T, const float *x, int32_t *meta, void *stream) {
    if (!m || !xc || !x || !meta || T < 1 || T > xc->Tmax || T > m->cfg.max_tokens)
        QE_FAIL("ep_route_p2p: bad arguments (T must be within the exchange's T_max and the handle's max_tokens)");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const int k = m->cfg.top_k, G = m->cfg.ep_size, E = m->cfg.E;
    const size_t H = m->cfg.hidden;
    if (ensure_ws(d, scratch_layout(m->cfg, T, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, T, (char *)d->ws, &sc);
    if (run_route(m, x, T, sc, s)) return -1;
    ep_meta_kernel<<<(T * k + 255) / 256, 256, 0, s>>>(sc.idx, sc.score, T, k, meta);
    QE_CHECK(cudaGetLastError());
    ep_gate_kernel<<<(T + 255) / 256, 256, 0, s>>>(sc.logits, T, E, (float *)(xc->mine + xc->off_gate));
    QE_CHECK(cudaGetLastError());
    QE_CHECK(cudaMemcpyAsync(xc->mine + (size_t)G * T * H * 4, x, sizeof(float) * (size_t)T * H,
                             cudaMemcpyDeviceToDevice, s));
    g_launches += 2;
    xc->fold_T = T;
    return 0;
}

int qe_moe_ep_experts_p2p(QeMoe *m, QeEpXchg *xc, int T, void *stream) {
    if (!m || !xc || T < 1 || T > xc->Tmax) QE_FAIL("ep_experts_p2p: bad arguments");
    DevCtx *d;
    if (dev_ctx(m->device, &d)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    const bool fold = xc->fold_T == T;
    const int G = m->cfg.ep_size, nr = G * T, n = nr + (fold ? T : 0), k = m->cfg.top_k;
    const int P = std::min(n, m->cfg.max_tokens);
    const size_t H = m->cfg.hidden;
    if (ensure_ws(d, scratch_layout(m->cfg, P, nullptr, nullptr))) return -1;
    Scratch sc;
    scratch_layout(m->cfg, P, (char *)d->ws, &sc);
    const float *rx = (const float *)xc->mine;
    const int32_t *rm = (const int32_t *)(xc->mine + xc->off_meta);
    const float *gate = (const float *)(xc->mine + xc->off_gate);
    float *sh_out = (float *)(xc->mine + xc->off_shared);
    for (int r0 = 0; r0 < n; r0 += P) {
        const int cnt = std::min(P, n - r0);
        const int cr = std::max(0, std::min(cnt, nr - r0));   /* received rows of this pass; the rest are own rows */
        if (cr > 0) {
            ep_local_kernel<<<(cr * k + 255) / 256, 256, 0, s>>>(rm + (size_t)r0 * 2 * k, cr, k, m->cfg.ep_rank,
                                                                place_of(m), sc.idx, sc.score);
            QE_CHECK(cudaGetLastError());
            g_launches += 1;
        }
        if (cnt > cr) QE_CHECK(cudaMemsetAsync(sc.idx + (size_t)cr * k, 0xff, sizeof(int32_t) * (size_t)(cnt - cr) * k, s));
        const EpScatter sca = {(float *const *)(xc->dptr + 2 * G), r0, T, m->cfg.ep_rank};
        const int o0 = r0 + cr - nr;                          /* first own row of this pass */
        const EpFold fo = {cr, cnt - cr, gate + std::max(0, o0), sh_out + (size_t)std::max(0, o0) * H};
        if (run_experts(m, rx + (size_t)r0 * H, nullptr, cnt, fold ? cr : cnt, sc, d->sms, true, false, s, &sca,
                        fold ? &fo : nullptr))
            return -1;
    }
    /* the partial rows written into the peers must be visible to them once this stream's work is done */
    return 0;
}

int qe_moe_ep_combine_p2p(QeMoe *m, QeEpXchg *xc, int T, const int32_t *home, const float *shared, float *out,
                          void *stream) {
    if (!xc || T < 1 || T > xc->Tmax) QE_FAIL("ep_combine_p2p: bad arguments");
    if (!shared) {
        /* the step was routed by qe_moe_ep_route_p2p: the shared-expert term is in the exchange */
        if (xc->fold_T != T) QE_FAIL("ep_combine_p2p: no shared term given and the step was not routed by "
                                     "qe_moe_ep_route_p2p");
        shared = (const float *)(xc->mine + xc->off_shared);
    }
    xc->fold_T = 0;
    return qe_moe_ep_combine_device(m, T, (const float *)(xc->mine + xc->off_back), home, shared, out, stream);
}

int qe_qmat_matvec(const uint32_t *w, const uint16_t *scales, const uint16_t *biases, int rows, int cols, int bits,
                   int group_size, const float *x, float *y) {
    /* validation exactly as engine/src/qmat.c:16-22 (y untouched on error) */
    if (!w || !scales || !biases || !x || !y) return -1;
    if (bits != 4 && bits != 8) return -1;
    if (group_size != 32 && group_size != 64 && group_size != 128) return -1;
    if (rows <= 0 || cols <= 0) return -1;
    if (cols % group_size != 0) return -1;
    if (cols / group_size > 4096) return -1;
    DevCtx *d;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev_ctx(dev, &d)) return -1;
    cudaStream_t s = d->stream;
    const size_t wb = (size_t)rows * ((size_t)cols * bits / 32) * 4, gb = (size_t)rows * (cols / group_size) * 2;
    char *buf = nullptr;
    const size_t total = align256(wb) + 2 * align256(gb) + align256(4 * (size_t)cols) + align256(4 * (size_t)rows);
    QE_CHECK(cudaMalloc((void **)&buf, total));
    QeQDev q;
    q.w = (const uint32_t *)buf;
    q.scales = (const uint16_t *)(buf + align256(wb));
    q.biases = (const uint16_t *)(buf + align256(wb) + align256(gb));
    float *dx = (float *)(buf + align256(wb) + 2 * align256(gb));
    float *dy = (float *)((char *)dx + align256(4 * (size_t)cols));
    q.rows = rows; q.cols = cols; q.bits = bits; q.group_size = group_size; q.scale_t = 0;
    int rc = cudaMemcpyAsync((void *)q.w, w, wb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
             cudaMemcpyAsync((void *)q.scales, scales, gb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
             cudaMemcpyAsync((void *)q.biases, biases, gb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
             cudaMemcpyAsync(dx, x, 4 * (size_t)cols, cudaMemcpyHostToDevice, s) != cudaSuccess;
    if (!rc) rc = qe_launch_qmatvec(&q, dx, 1, dy, s);
    if (!rc) rc = cudaMemcpyAsync(y, dy, 4 * (size_t)rows, cudaMemcpyDeviceToHost, s) != cudaSuccess;
    if (!rc) rc = cudaStreamSynchronize(s) != cudaSuccess;
    cudaFree(buf);
    return rc ? -1 : 0;
}

int qe_route_logits(int T, int E, int k, const float *logits, float *probs, int32_t *idx, float *score) {
    if (T < 1 || !logits || !idx || !score) return -1;
    if (E < 1 || E > 512 || k < 1 || k > 16 || k > E) return -1;
    DevCtx *d;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev_ctx(dev, &d)) return -1;
    cudaStream_t s = d->stream;
    char *buf = nullptr;
    const size_t lb = align256(4 * (size_t)T * E), kb = align256(4 * (size_t)T * k);
    QE_CHECK(cudaMalloc((void **)&buf, 2 * lb + 2 * kb));
    float *dl = (float *)buf, *dp = (float *)(buf + lb), *ds = (float *)(buf + 2 * lb);
    int32_t *di = (int32_t *)(buf + 2 * lb + kb);
    int rc = cudaMemcpyAsync(dl, logits, 4 * (size_t)T * E, cudaMemcpyHostToDevice, s) != cudaSuccess;
    if (!rc) rc = qe_launch_route_topk(dl, E, T, E, k, di, ds, dp, s);
    if (!rc && probs) rc = cudaMemcpyAsync(probs, dp, 4 * (size_t)T * E, cudaMemcpyDeviceToHost, s) != cudaSuccess;
    if (!rc) rc = cudaMemcpyAsync(idx, di, 4 * (size_t)T * k, cudaMemcpyDeviceToHost, s) != cudaSuccess;
    if (!rc) rc = cudaMemcpyAsync(score, ds, 4 * (size_t)T * k, cudaMemcpyDeviceToHost, s) != cudaSuccess;
    if (!rc) rc = cudaStreamSynchronize(s) != cudaSuccess;
    cudaFree(buf);
    return rc ? -1 : 0;
}

static int run_op(int op, float *out, const float *a, const float *b, int n) {
    if (n < 1 || !out || !a || (op == 0 && !b)) return -1;
    DevCtx *d;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev_ctx(dev, &d)) return -1;
    cudaStream_t s = d->stream;
    float *buf = nullptr;
    const size_t nb = align256(4 * (size_t)n);
    QE_CHECK(cudaMalloc((void **)&buf, 3 * nb));
    float *da = buf, *db = (float *)((char *)buf + nb), *dout = (float *)((char *)buf + 2 * nb);
    int rc = cudaMemcpyAsync(da, a, 4 * (size_t)n, cudaMemcpyHostToDevice, s) != cudaSuccess;
    if (!rc && op == 0) rc = cudaMemcpyAsync(db, b, 4 * (size_t)n, cudaMemcpyHostToDevice, s) != cudaSuccess;
    if (!rc) {
        ops_kernel<<<(n + 255) / 256, 256, 0, s>>>(op, da, db, dout, n);
        rc = cudaGetLastError() != cudaSuccess;
    }
    if (!rc) rc = cudaMemcpyAsync(out, dout, 4 * (size_t)n, cudaMemcpyDeviceToHost, s) != cudaSuccess;
    if (!rc) rc = cudaStreamSynchronize(s) != cudaSuccess;
    cudaFree(buf);
    return rc ? -1 : 0;
}

int qe_op_silu_mul(float *out, const float *gate, const float *up, int n) { return run_op(0, out, gate, up, n); }
int qe_op_sigmoid(float *out, const float *x, int n) { return run_op(1, out, x, nullptr, n); }
int qe_op_expf(float *out, const float *x, int n) { return run_op(2, out, x, nullptr, n); }

int qe_profile_begin(int device) {
    if (device < 0 || device >= 64) return -1;
    g_prof[device].on = true;
    g_prof[device].used = 0;
    return 0;
}

int qe_profile_end(int device, double *stage_ms, int *passes) {
    if (device < 0 || device >= 64) return -1;
    Prof &p = g_prof[device];
    p.on = false;
    for (int i = 0; i < kStages; i++) stage_ms[i] = 0.0;
    const size_t per = kStages + 1;
    const size_t n = p.used / per;
    QE_CHECK(cudaSetDevice(device));
    for (size_t k = 0; k < n; k++) {
        QE_CHECK(cudaEventSynchronize(p.pool[k * per + kStages]));
        for (int i = 0; i < kStages; i++) {
            float ms = 0.0f;
            QE_CHECK(cudaEventElapsedTime(&ms, p.pool[k * per + i], p.pool[k * per + i + 1]));
            stage_ms[i] += ms;
        }
    }
    if (passes) *passes = (int)n;
    p.used = 0;
    return 0;
}

unsigned long long qe_kernel_launches(void) { return g_launches.load(); }
unsigned long long qe_graph_captures(void) { return g_captures.load(); }

int qe_device_error(void) {
    const int t = qe_tc_error(), d = qe_decode_error();
    int e = 0;
    if (cudaMemcpyFromSymbol(&e, g_ep_error, sizeof(int)) != cudaSuccess) return -1;
    return t ? t : d ? 100 + d : e ? 200 + e : 0;
}

int qe_device_error_on(int device) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) return -1;
    const int e = qe_device_error();
    cudaSetDevice(cur);
    return e;
}

int qe_device_error_reset(int device) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return -1;
    QE_CHECK(cudaSetDevice(device));
    const int zero = 0;
    const int rc = qe_tc_error_reset() || qe_decode_error_reset() ||
                   cudaMemcpyToSymbol(g_ep_error, &zero, sizeof(int)) != cudaSuccess;
    cudaSetDevice(cur);
    return rc ? -1 : 0;
}

int qe_ep_xchg_set_timeout_ms(QeEpXchg *x, int ms) {
    if (!x || ms < 1 || ms > 60000) QE_FAIL("ep_xchg_set_timeout_ms: bad arguments");
    x->wait_ns = (unsigned long long)ms * 1000000ull;
    return 0;
}

double qe_expert_gb_read(void) { return (double)g_bytes_read.load() / 1e9; }

int qe_set_threads(int n) {
    if (n > 0) g_host_threads.store(n);
    return host_threads();
}

}  // extern "C"

int qe_host_thread_count(void) { return host_threads(); }

extern "C" {

double qe_peak_rss_gb(void) {
    struct rusage ru;
    if (getrusage(RUSAGE_SELF, &ru)) return -1.0;
    return (double)ru.ru_maxrss * 1024.0 / 1073741824.0;   /* ru_maxrss: KiB on Linux */
}
double qe_expert_read_seconds(void) { return g_gpu_seconds; }
int qe_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

}  // extern "C"
