/* engine.cu: the whole-model ABI (include/qe_engine.h) over the GPU MoE blocks.
 *
 * The reference engine runs a qwen3_5_moe MLX checkpoint one token at a time on the CPU
 * (engine/src/model.c:135-157, front-end API engine/src/qengine.c:12-47). Here the routed MoE block of every
 * layer is a libqengine_b200 handle (experts resident in HBM, the GPU kernels of this library); the trunk
 * around it -- embedding row, RMSNorms, Gated DeltaNet and gated full-attention layers, residuals, final norm
 * and LM head -- is fp32 host code on a pool of qe_set_threads threads, reading the checkpoint's trunk tensors
 * in place from its memory mappings. The trunk follows the contracts the reference documents for its ops
 * (engine/include/ops.h, gdn.h, gdn_layer.h, attn_layer.h; the Qwen3.5 / Qwen3-Next architecture):
 *   RMSNorm      out = x / sqrt(mean(x^2) + eps) * w, the square sum in double
 *   RoPE         rotate-half on the first rot_dims of each head, angle pos * theta^(-2i/rot_dims) in double
 *   GDN layer    qkv/z/a/b projections, causal depthwise conv + SiLU, per-head L2 norms (q scaled by
 *                1/sqrt(Dk)), gates g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b), the delta
 *                rule S = g S; S += k (beta (v - S k))^T; y = S q, gated RMSNorm y * silu(z), out projection
 *   attention    q (with a per-head output gate), k, v projections, per-head RMSNorm of q and k, RoPE, KV
 *                cache, causal softmax attention (exp and sum in double), sigmoid(gate) * att, out projection
 *   quantized    y[r] = sum over groups of scale * sum_q + bias * sum_x (MLX affine, qmat.c:36-46 semantics)
 * Results match the reference's within fp32 reordering (tests/test_gpu_engine.py against the reference's own
 * qe_forward on a synthetic checkpoint).
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <condition_variable>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>

#include "ckpt.h"
#include "qe_kernels.h"
#include "trunk.h"
#include "../../include/qe_engine.h"

using namespace qe_ckpt;

namespace {

/* ------------------------------------------------------------------ thread pool */

/* Workers that split an index range [0, n) in chunks; the calling thread works too. Sized from
 * qe_set_threads at each call (resized when the count changes). One job at a time. */
class Pool {
public:
    ~Pool() { resize(0); }

    void parallel_for(int n, int grain, const std::function<void(int, int)> &fn) {
        const int want = std::max(1, qe_host_thread_count());
        const int chunks = (n + grain - 1) / grain;
        if (want == 1 || chunks <= 1) {
            fn(0, n);
            return;
        }
        if ((int)workers_.size() != want - 1) resize(want - 1);
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &fn;
            n_ = n;
            grain_ = grain;
            next_.store(0);
            active_ = (int)workers_.size();
            gen_++;
        }
        cv_.notify_all();
        work();
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [&] { return active_ == 0; });
        job_ = nullptr;
    }

private:
    void work() {
        while (true) {
            const int a = next_.fetch_add(grain_);
            if (a >= n_) break;
            (*job_)(a, std::min(n_, a + grain_));
        }
    }
    void loop(uint64_t seen) {   /* seen: the job generation current when the worker started */
        while (true) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
            }
            work();
            std::lock_guard<std::mutex> lk(mu_);
            if (--active_ == 0) done_.notify_one();
        }
    }
    void resize(int n) {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
        workers_.clear();
        stop_ = false;
        const uint64_t g = gen_;
        for (int i = 0; i < n; i++) workers_.emplace_back([this, g] { loop(g); });
    }

    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::function<void(int, int)> *job_ = nullptr;
    int n_ = 0, grain_ = 1, active_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
    std::atomic<int> next_{0};
};

Pool &pool() {
    static Pool p;
    return p;
}

/* ------------------------------------------------------------------ JSON (config.json) */

struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal *get(const char *k) const {
        if (kind != OBJ) return nullptr;
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char *p, *end;
    int depth = 0;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
    }
    bool string(std::string &out) {
        if (p >= end || *p != '"') return false;
        p++;
        out.clear();
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return false;
                const char e = *p++;
                switch (e) {
                case 'n': c = '\n'; break;
                case 't': c = '\t'; break;
                case 'r': c = '\r'; break;
                case 'b': c = '\b'; break;
                case 'f': c = '\f'; break;
                case 'u':   /* keys and values the engine reads are ASCII: keep a placeholder */
                    if (end - p < 4) return false;
                    p += 4;
                    c = '?';
                    break;
                default: c = e;
                }
            }
            out += c;
        }
        if (p >= end) return false;
        p++;
        return true;
    }
    bool value(JVal &v) {
        ws();
        if (p >= end || ++depth > 64) return false;
        bool ok = true;
        if (*p == '{') {
            v.kind = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') {
                p++;
            } else {
                while (ok) {
                    ws();
                    std::string k;
                    JVal x;
                    ok = string(k);
                    ws();
                    ok = ok && p < end && *p++ == ':' && value(x);
                    if (!ok) break;
                    v.obj.emplace_back(std::move(k), std::move(x));
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    ok = p < end && *p++ == '}';
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') {
                p++;
            } else {
                while (ok) {
                    JVal x;
                    ok = value(x);
                    if (!ok) break;
                    v.arr.push_back(std::move(x));
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    ok = p < end && *p++ == ']';
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = JVal::STR;
            ok = string(v.str);
        } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
            v.kind = JVal::BOOL, v.b = true, p += 4;
        } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
            v.kind = JVal::BOOL, v.b = false, p += 5;
        } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
            v.kind = JVal::NUL, p += 4;
        } else {
            char *q = nullptr;
            std::string tok;
            while (p < end && (isdigit((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.' || *p == 'e' || *p == 'E'))
                tok += *p++;
            v.kind = JVal::NUM;
            v.num = strtod(tok.c_str(), &q);
            ok = !tok.empty() && q && *q == '\0';
        }
        depth--;
        return ok;
    }
};

/* ------------------------------------------------------------------ configuration */

struct Cfg {
    int hidden, n_layers, vocab, full_attn_interval;
    int Hq, Hkv, head_dim, rot_dims;
    float rope_theta;
    int lin_Hk, lin_Hv, lin_Dk, lin_Dv, conv_K;
    int E, top_k, moe_inter, sh_inter;
    float eps;
    int group_size;
};

int read_config(const char *dir, Cfg &c) {
    const std::string path = std::string(dir) + "/config.json";
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) QE_FAIL("engine: cannot open %s", path.c_str());
    std::string text;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
    fclose(f);
    JVal root;
    JParser jp{text.data(), text.data() + text.size()};
    if (!jp.value(root) || root.kind != JVal::OBJ) QE_FAIL("engine: %s is not a JSON object", path.c_str());
    const JVal *t = root.get("text_config");
    if (!t) t = &root;
    const JVal *q = root.get("quantization");
    bool ok = true;
    auto num = [&](const JVal *o, const char *k, double &out) {
        const JVal *v = o ? o->get(k) : nullptr;
        if (!v || v->kind != JVal::NUM) {
            if (ok) fprintf(stderr, "qengine_b200: config: missing or non-numeric \"%s\"\n", k);
            ok = false;
            return;
        }
        out = v->num;
    };
    auto ival = [&](const JVal *o, const char *k, int &out) { double d = 0; num(o, k, d); out = (int)d; };
    auto fval = [&](const JVal *o, const char *k, float &out) { double d = 0; num(o, k, d); out = (float)d; };
    ival(t, "hidden_size", c.hidden);
    ival(t, "num_hidden_layers", c.n_layers);
    ival(t, "vocab_size", c.vocab);
    ival(t, "full_attention_interval", c.full_attn_interval);
    ival(t, "num_attention_heads", c.Hq);
    ival(t, "num_key_value_heads", c.Hkv);
    ival(t, "head_dim", c.head_dim);
    ival(t, "linear_num_key_heads", c.lin_Hk);
    ival(t, "linear_num_value_heads", c.lin_Hv);
    ival(t, "linear_key_head_dim", c.lin_Dk);
    ival(t, "linear_value_head_dim", c.lin_Dv);
    ival(t, "linear_conv_kernel_dim", c.conv_K);
    ival(t, "num_experts", c.E);
    ival(t, "num_experts_per_tok", c.top_k);
    ival(t, "moe_intermediate_size", c.moe_inter);
    ival(t, "shared_expert_intermediate_size", c.sh_inter);
    fval(t, "rms_norm_eps", c.eps);
    if (!ok) return -1;
    if (!q) QE_FAIL("engine: config: no \"quantization\" object (not an MLX quantized checkpoint)");
    ival(q, "group_size", c.group_size);
    if (!ok) return -1;
    const JVal *mode = q->get("mode");
    if (mode && (mode->kind != JVal::STR || mode->str != "affine")) QE_FAIL("engine: config: only affine quantization");
    const JVal *mt = t->get("model_type");
    if (!mt || mt->kind != JVal::STR || mt->str.compare(0, 11, "qwen3_5_moe"))
        QE_FAIL("engine: config: model_type must be qwen3_5_moe*, got %s",
                mt && mt->kind == JVal::STR ? mt->str.c_str() : "?");
    const JVal *nt = t->get("norm_topk_prob");
    if (nt && nt->kind == JVal::BOOL && !nt->b) QE_FAIL("engine: config: norm_topk_prob=false is not supported");
    const JVal *rp = t->get("rope_parameters");
    if (!rp || rp->kind != JVal::OBJ) QE_FAIL("engine: config: no \"rope_parameters\" object");
    const JVal *rt = rp->get("rope_type");
    if (rt && (rt->kind != JVal::STR || rt->str != "default")) QE_FAIL("engine: config: only rope_type \"default\"");
    float partial = 0;
    fval(rp, "partial_rotary_factor", partial);
    fval(rp, "rope_theta", c.rope_theta);
    if (!ok) return -1;
    c.rot_dims = (int)(c.head_dim * partial);
    if (c.rot_dims <= 0 || c.rot_dims % 2 || c.rot_dims > c.head_dim) QE_FAIL("engine: config: bad partial rotary factor");
    if (c.hidden <= 0 || c.n_layers <= 0 || c.vocab <= 0 || c.full_attn_interval < 1 || c.Hq <= 0 || c.Hkv <= 0 ||
        c.Hq % c.Hkv || c.lin_Hk <= 0 || c.lin_Hv % c.lin_Hk || c.lin_Dk <= 0 || c.lin_Dv <= 0 || c.conv_K < 2 ||
        c.top_k < 1 || c.top_k > 16 || c.E < c.top_k)
        QE_FAIL("engine: config: unsupported head/expert layout");
    return 0;
}

/* ------------------------------------------------------------------ host tensors */

float bf16f(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float f16f(uint16_t h) {   /* IEEE binary16 -> binary32 */
    const uint32_t sign = (uint32_t)(h >> 15) << 31, ex = (h >> 10) & 31, man = h & 1023;
    float f;
    if (ex == 0) {
        f = ldexpf((float)man, -24);
        return sign ? -f : f;
    }
    const uint32_t u = ex == 31 ? sign | 0x7f800000u | (man << 13) : sign | ((ex + 112) << 23) | (man << 13);
    memcpy(&f, &u, 4);
    return f;
}

/* One MLX affine quantized matrix read in place from the checkpoint (engine/include/qmat.h:3-11). */
struct HQ {
    const uint32_t *w = nullptr;
    const uint16_t *s = nullptr, *b = nullptr;
    int rows = 0, cols = 0, bits = 0, gs = 0;
};

int load_hq(const Checkpoint &ck, const std::string &base, int gs, HQ &m) {
    QView v;
    if (qview(ck, base, 2, v)) return -1;
    m.cols = (int)(v.groups * gs);
    m.bits = m.cols ? (int)(v.packed * 32 / m.cols) : 0;
    if ((m.bits != 4 && m.bits != 8) || v.packed * 32 != (int64_t)m.bits * m.cols)
        QE_FAIL("engine: %s: cannot derive 4/8 bits from %lld packed words and %d columns", base.c_str(),
                (long long)v.packed, m.cols);
    m.w = v.t.w;
    m.s = v.t.scales;
    m.b = v.t.biases;
    m.rows = (int)v.rows;
    m.gs = gs;
    return 0;
}

int load_vec(const Checkpoint &ck, const std::string &name, std::vector<float> &out, int64_t want = -1) {
    const TensorInfo *t = ck.find(name);
    if (!t) QE_FAIL("engine: missing %s", name.c_str());
    int64_t n = 1;
    for (int64_t d : t->shape) n *= d;
    if (want >= 0 && n != want) QE_FAIL("engine: %s has %lld elements, expected %lld", name.c_str(), (long long)n,
                                        (long long)want);
    out.resize((size_t)n);
    const void *p = ck.data(*t);
    if (t->dtype == "F32") {
        memcpy(out.data(), p, sizeof(float) * (size_t)n);
    } else if (t->dtype == "BF16" || t->dtype == "F16") {
        const bool bf = t->dtype == "BF16";
        for (int64_t i = 0; i < n; i++) {
            uint16_t h;
            memcpy(&h, (const char *)p + 2 * i, 2);
            out[(size_t)i] = bf ? bf16f(h) : f16f(h);
        }
    } else {
        QE_FAIL("engine: %s: dtype %s (F32, BF16 or F16 expected)", name.c_str(), t->dtype.c_str());
    }
    return 0;
}

inline uint32_t code(const uint32_t *row, int j, int bits) {
    return bits == 4 ? (row[j >> 3] >> ((j & 7) * 4)) & 15u : (row[j >> 2] >> ((j & 3) * 8)) & 255u;
}

/* y = W x: per row, groups in order, acc += scale * sum_q + bias * sum_x (qmat.c:36-46 semantics); rows on the
 * pool. gsum: cols / gs floats of scratch. */
void hq_matvec(const HQ &m, const float *x, float *y, std::vector<float> &gsum) {
    const int ng = m.cols / m.gs, wpr = m.cols * m.bits / 32;
    gsum.resize((size_t)ng);
    for (int g = 0; g < ng; g++) {
        float s = 0.0f;
        for (int j = 0; j < m.gs; j++) s += x[g * m.gs + j];
        gsum[(size_t)g] = s;
    }
    const float *gs = gsum.data();
    pool().parallel_for(m.rows, 64, [&](int r0, int r1) {
        for (int r = r0; r < r1; r++) {
            const uint32_t *row = m.w + (size_t)r * wpr;
            const uint16_t *sr = m.s + (size_t)r * ng, *br = m.b + (size_t)r * ng;
            float acc = 0.0f;
            for (int g = 0; g < ng; g++) {
                float sq = 0.0f;
                const int j0 = g * m.gs;
                for (int j = 0; j < m.gs; j++) sq += (float)code(row, j0 + j, m.bits) * x[j0 + j];
                acc += bf16f(sr[g]) * sq + bf16f(br[g]) * gs[g];
            }
            y[r] = acc;
        }
    });
}

/* Row r of W dequantized (the embedding lookup, qmat_row.c semantics): out[c] = q * scale + bias. */
int hq_row(const HQ &m, int r, float *out) {
    if (r < 0 || r >= m.rows) return -1;
    const int ng = m.cols / m.gs, wpr = m.cols * m.bits / 32;
    const uint32_t *row = m.w + (size_t)r * wpr;
    for (int c = 0; c < m.cols; c++) {
        const int g = c / m.gs;
        out[c] = (float)code(row, c, m.bits) * bf16f(m.s[(size_t)r * ng + g]) + bf16f(m.b[(size_t)r * ng + g]);
    }
    return 0;
}

float silu(float v) { return v / (1.0f + expf(-v)); }
float sigmoidf(float v) { return 1.0f / (1.0f + expf(-v)); }

/* ------------------------------------------------------------------ the model */

struct GdnLayer {
    HQ qkv, z, a, b, out;
    std::vector<float> conv_w, A_log, dt_bias, norm_w;
    std::vector<float> conv_state, rec_state;
};

struct AttnLayer {
    HQ q, k, v, o;
    std::vector<float> q_norm, k_norm;
    std::vector<float> kc, vc;   /* [max_len][Hkv * D] keys after norm and RoPE, values */
    int len = 0;
};

struct Layer {
    bool linear = false;
    std::vector<float> in_norm, post_norm;
    GdnLayer g;
    AttnLayer a;
    QeMoe *moe = nullptr;
};

}  // namespace

struct QeModel {
    Cfg c{};
    Checkpoint ck;
    HQ embed, lm_head;
    std::vector<float> final_norm;
    std::vector<Layer> layers;
    std::vector<float> x, h, t1, t2, gsum;
    std::vector<float> s1, s2, s3, s4, s5, s6;   /* per-layer scratch */
    int max_len = 0, pos = 0;
    GpuTrunk *gt = nullptr;   /* the trunk on the GPU (default), or null: the host trunk (QE_TRUNK=host) */
    ~QeModel() {
        if (gt) qe_gtrunk_free(gt);
        for (auto &L : layers)
            if (L.moe) qe_moe_free(L.moe);
    }
};

namespace {

void rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float r = (float)sqrt(ss / n + (double)eps);
    for (int i = 0; i < n; i++) out[i] = x[i] / r * w[i];
}

void rope(float *x, int n_heads, int D, int rot, int pos, float theta) {
    const int half = rot / 2;
    for (int i = 0; i < half; i++) {
        const double ang = (double)pos * pow((double)theta, -2.0 * i / rot);
        const float cs = (float)cos(ang), sn = (float)sin(ang);
        for (int h = 0; h < n_heads; h++) {
            float *v = x + (size_t)h * D;
            const float a = v[i], b = v[i + half];
            v[i] = a * cs - b * sn;
            v[i + half] = b * cs + a * sn;
        }
    }
}

void conv_step(float *out, float *state, const float *x, const float *w, int C, int K) {
    for (int c = 0; c < C; c++) {
        float acc = 0.0f;
        for (int j = 0; j + 1 < K; j++) acc += state[(size_t)j * C + c] * w[(size_t)c * K + j];
        acc += w[(size_t)c * K + K - 1] * x[c];
        out[c] = silu(acc);
    }
    /* the window moves by one input: rows 1..K-2 up, x into the last row */
    if (K > 2) memmove(state, state + C, sizeof(float) * (size_t)(K - 2) * C);
    memcpy(state + (size_t)(K - 2) * C, x, sizeof(float) * C);
}

void l2norm(float *v, int n, float eps, float scale) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)v[i] * (double)v[i];
    const float f = (float)(scale / sqrt(ss + (double)eps));
    for (int i = 0; i < n; i++) v[i] *= f;
}

void gates(float *g, float *beta, const float *a, const float *b, const float *A_log, const float *dt_bias, int Hv) {
    for (int h = 0; h < Hv; h++) {
        const float t = a[h] + dt_bias[h];
        const float sp = t > 20.0f ? t : logf(1.0f + expf(t));
        g[h] = expf(-expf(A_log[h]) * sp);
        beta[h] = sigmoidf(b[h]);
    }
}

void recurrent_step(float *y, float *state, const float *q, const float *k, const float *v, const float *g,
                    const float *beta, int Hk, int Hv, int Dk, int Dv) {
    const int per = Hv / Hk;
    pool().parallel_for(Hv * Dv, 16, [&](int i0, int i1) {
        for (int hi = i0; hi < i1; hi++) {
            const int h = hi / Dv, i = hi % Dv, kh = h / per;
            const float *kk = k + (size_t)kh * Dk, *kq = q + (size_t)kh * Dk;
            float *S = state + ((size_t)h * Dv + i) * Dk;
            float kv = 0.0f;
            for (int j = 0; j < Dk; j++) {
                S[j] *= g[h];
                kv += S[j] * kk[j];
            }
            const float d = (v[(size_t)h * Dv + i] - kv) * beta[h];
            float o = 0.0f;
            for (int j = 0; j < Dk; j++) {
                S[j] += kk[j] * d;
                o += S[j] * kq[j];
            }
            y[(size_t)h * Dv + i] = o;
        }
    });
}

int gdn_forward(QeModel *m, Layer &L, const float *x, float *out) {
    const Cfg &c = m->c;
    GdnLayer &G = L.g;
    const int KD = c.lin_Hk * c.lin_Dk, VD = c.lin_Hv * c.lin_Dv, C = 2 * KD + VD;
    float *qkv = m->s1.data(), *cv = m->s2.data(), *z = m->s3.data(), *y = m->s4.data(), *a = m->s5.data(),
          *b = m->s5.data() + c.lin_Hv, *g = m->s5.data() + 2 * c.lin_Hv, *beta = m->s5.data() + 3 * c.lin_Hv;
    hq_matvec(G.qkv, x, qkv, m->gsum);
    hq_matvec(G.z, x, z, m->gsum);
    hq_matvec(G.a, x, a, m->gsum);
    hq_matvec(G.b, x, b, m->gsum);
    conv_step(cv, G.conv_state.data(), qkv, G.conv_w.data(), C, c.conv_K);
    for (int h = 0; h < c.lin_Hk; h++) {
        l2norm(cv + (size_t)h * c.lin_Dk, c.lin_Dk, 1e-6f, 1.0f / sqrtf((float)c.lin_Dk));
        l2norm(cv + KD + (size_t)h * c.lin_Dk, c.lin_Dk, 1e-6f, 1.0f);
    }
    gates(g, beta, a, b, G.A_log.data(), G.dt_bias.data(), c.lin_Hv);
    recurrent_step(y, G.rec_state.data(), cv, cv + KD, cv + 2 * KD, g, beta, c.lin_Hk, c.lin_Hv, c.lin_Dk, c.lin_Dv);
    float *nrm = m->s6.data();
    for (int h = 0; h < c.lin_Hv; h++) {
        float *yh = y + (size_t)h * c.lin_Dv;
        const float *zh = z + (size_t)h * c.lin_Dv;
        rmsnorm(nrm, yh, G.norm_w.data(), c.lin_Dv, c.eps);
        for (int i = 0; i < c.lin_Dv; i++) yh[i] = silu(zh[i]) * nrm[i];
    }
    hq_matvec(G.out, y, out, m->gsum);
    return 0;
}

int attn_forward(QeModel *m, Layer &L, const float *x, float *out) {
    const Cfg &c = m->c;
    AttnLayer &A = L.a;
    const int D = c.head_dim, QD = c.Hq * D, KD = c.Hkv * D, pos = A.len;
    if (pos >= m->max_len) return -2;
    float *qg = m->s1.data(), *q = m->s2.data(), *att = m->s3.data(), *kx = m->s4.data(), *vx = m->s5.data(),
          *sc = m->s6.data();
    hq_matvec(A.q, x, qg, m->gsum);
    hq_matvec(A.k, x, kx, m->gsum);
    hq_matvec(A.v, x, vx, m->gsum);
    for (int h = 0; h < c.Hq; h++) rmsnorm(q + (size_t)h * D, qg + (size_t)h * 2 * D, A.q_norm.data(), D, c.eps);
    float *kn = A.kc.data() + (size_t)pos * KD;
    for (int h = 0; h < c.Hkv; h++) rmsnorm(kn + (size_t)h * D, kx + (size_t)h * D, A.k_norm.data(), D, c.eps);
    rope(q, c.Hq, D, c.rot_dims, pos, c.rope_theta);
    rope(kn, c.Hkv, D, c.rot_dims, pos, c.rope_theta);
    memcpy(A.vc.data() + (size_t)pos * KD, vx, sizeof(float) * KD);
    const int n = pos + 1, per = c.Hq / c.Hkv;
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    pool().parallel_for(c.Hq, 1, [&](int h0, int h1) {
        for (int h = h0; h < h1; h++) {
            const int kvh = h / per;
            const float *qh = q + (size_t)h * D;
            float *s = sc + (size_t)h * m->max_len;
            float mx = -INFINITY;
            for (int t = 0; t < n; t++) {
                const float *kt = A.kc.data() + (size_t)t * KD + (size_t)kvh * D;
                float d = 0.0f;
                for (int i = 0; i < D; i++) d += qh[i] * kt[i];
                s[t] = d * inv_sqrt_d;
                mx = fmaxf(mx, s[t]);
            }
            double sum = 0.0;
            for (int t = 0; t < n; t++) sum += exp((double)s[t] - (double)mx);
            for (int t = 0; t < n; t++) s[t] = (float)(exp((double)s[t] - (double)mx) / sum);
            float *ah = att + (size_t)h * D;
            const float *gate = qg + (size_t)h * 2 * D + D;
            for (int i = 0; i < D; i++) {
                float o = 0.0f;
                for (int t = 0; t < n; t++) o += s[t] * A.vc[(size_t)t * KD + (size_t)kvh * D + i];
                ah[i] = o * sigmoidf(gate[i]);
            }
        }
    });
    A.len = pos + 1;
    (void)QD;
    hq_matvec(A.o, att, out, m->gsum);
    return 0;
}

int load_model(QeModel *m, const char *dir, int max_len) {
    Cfg &c = m->c;
    if (read_config(dir, c)) return -1;
    if (m->ck.open_dir(dir)) return -1;
    m->max_len = max_len;
    const std::string P = "language_model.model.layers.";
    if (load_hq(m->ck, "language_model.model.embed_tokens", c.group_size, m->embed) ||
        load_hq(m->ck, "language_model.lm_head", c.group_size, m->lm_head) ||
        load_vec(m->ck, "language_model.model.norm.weight", m->final_norm, c.hidden))
        return -1;
    if (m->embed.cols != c.hidden || m->embed.rows != c.vocab || m->lm_head.cols != c.hidden || m->lm_head.rows != c.vocab)
        QE_FAIL("engine: embedding / LM head shapes do not match hidden %d and vocab %d", c.hidden, c.vocab);
    const int KD = c.lin_Hk * c.lin_Dk, VD = c.lin_Hv * c.lin_Dv, C = 2 * KD + VD;
    int dev = 0;
    if (const char *e = getenv("QE_DEVICE")) dev = atoi(e);
    m->layers.resize((size_t)c.n_layers);
    for (int l = 0; l < c.n_layers; l++) {
        Layer &L = m->layers[(size_t)l];
        const std::string b = P + std::to_string(l) + ".";
        L.linear = (l + 1) % c.full_attn_interval != 0;
        if (load_vec(m->ck, b + "input_layernorm.weight", L.in_norm, c.hidden) ||
            load_vec(m->ck, b + "post_attention_layernorm.weight", L.post_norm, c.hidden))
            return -1;
        if (L.linear) {
            GdnLayer &G = L.g;
            const std::string f = b + "linear_attn.";
            if (load_hq(m->ck, f + "in_proj_qkv", c.group_size, G.qkv) || load_hq(m->ck, f + "in_proj_z", c.group_size, G.z) ||
                load_hq(m->ck, f + "in_proj_a", c.group_size, G.a) || load_hq(m->ck, f + "in_proj_b", c.group_size, G.b) ||
                load_hq(m->ck, f + "out_proj", c.group_size, G.out) ||
                load_vec(m->ck, f + "conv1d.weight", G.conv_w, (int64_t)C * c.conv_K) ||
                load_vec(m->ck, f + "A_log", G.A_log, c.lin_Hv) || load_vec(m->ck, f + "dt_bias", G.dt_bias, c.lin_Hv) ||
                load_vec(m->ck, f + "norm.weight", G.norm_w, c.lin_Dv))
                return -1;
            if (G.qkv.rows != C || G.z.rows != VD || G.a.rows != c.lin_Hv || G.b.rows != c.lin_Hv || G.out.cols != VD ||
                G.out.rows != c.hidden || G.qkv.cols != c.hidden)
                QE_FAIL("engine: layer %d: linear-attention shapes do not match the config", l);
            G.conv_state.assign((size_t)(c.conv_K - 1) * C, 0.0f);
            G.rec_state.assign((size_t)c.lin_Hv * c.lin_Dv * c.lin_Dk, 0.0f);
        } else {
            AttnLayer &A = L.a;
            const std::string f = b + "self_attn.";
            const int D = c.head_dim;
            if (load_hq(m->ck, f + "q_proj", c.group_size, A.q) || load_hq(m->ck, f + "k_proj", c.group_size, A.k) ||
                load_hq(m->ck, f + "v_proj", c.group_size, A.v) || load_hq(m->ck, f + "o_proj", c.group_size, A.o) ||
                load_vec(m->ck, f + "q_norm.weight", A.q_norm, D) || load_vec(m->ck, f + "k_norm.weight", A.k_norm, D))
                return -1;
            if (A.q.rows != 2 * c.Hq * D || A.k.rows != c.Hkv * D || A.v.rows != c.Hkv * D || A.o.cols != c.Hq * D ||
                A.o.rows != c.hidden)
                QE_FAIL("engine: layer %d: attention shapes do not match the config", l);
            A.kc.assign((size_t)max_len * c.Hkv * D, 0.0f);
            A.vc.assign((size_t)max_len * c.Hkv * D, 0.0f);
        }
        QeMoeConfig mc{};
        mc.hidden = c.hidden;
        mc.E = c.E;
        mc.top_k = c.top_k;
        mc.inter = c.moe_inter;
        mc.sh_inter = c.sh_inter;
        mc.group_size = c.group_size;
        mc.max_tokens = 16;
        mc.device = dev;
        mc.layer = l;
        L.moe = qe_moe_open_safetensors(dir, (b + "mlp").c_str(), &mc);
        if (!L.moe) QE_FAIL("engine: layer %d: MoE block not loaded", l);
    }
    const size_t H = (size_t)c.hidden, QD = (size_t)c.Hq * c.head_dim, KVD = (size_t)c.Hkv * c.head_dim;
    const size_t big = std::max<size_t>({(size_t)C, 2 * QD, H, (size_t)VD});
    m->x.assign(H, 0.0f);
    m->h.assign(H, 0.0f);
    m->t1.assign(H, 0.0f);
    m->t2.assign(H, 0.0f);
    m->s1.assign(big, 0.0f);
    m->s2.assign(big, 0.0f);
    m->s3.assign(big, 0.0f);
    m->s4.assign(std::max<size_t>(big, KVD), 0.0f);
    m->s5.assign(std::max<size_t>((size_t)4 * c.lin_Hv, KVD), 0.0f);
    m->s6.assign(std::max<size_t>((size_t)c.Hq * max_len, (size_t)c.lin_Dv), 0.0f);
    /* the trunk on the GPU, beside the MoE blocks, unless QE_TRUNK=host */
    const char *tr = getenv("QE_TRUNK");
    if (!tr || strcmp(tr, "host") != 0) {
        auto hq = [](const HQ &q) {
            TkHostQ t;
            t.w = q.w; t.s = q.s; t.b = q.b; t.rows = q.rows; t.cols = q.cols; t.bits = q.bits; t.gs = q.gs;
            return t;
        };
        TkDims d{};
        d.hidden = c.hidden; d.vocab = c.vocab; d.Hq = c.Hq; d.Hkv = c.Hkv; d.D = c.head_dim; d.rot = c.rot_dims;
        d.lin_Hk = c.lin_Hk; d.lin_Hv = c.lin_Hv; d.lin_Dk = c.lin_Dk; d.lin_Dv = c.lin_Dv; d.conv_K = c.conv_K;
        d.max_len = max_len; d.eps = c.eps; d.theta = c.rope_theta;
        std::vector<TkLayerHost> lh(m->layers.size());
        for (size_t l = 0; l < m->layers.size(); l++) {
            const Layer &L = m->layers[l];
            TkLayerHost &h = lh[l];
            h.linear = L.linear;
            h.in_norm = L.in_norm.data();
            h.post_norm = L.post_norm.data();
            h.moe = L.moe;
            if (L.linear) {
                h.qkv = hq(L.g.qkv); h.z = hq(L.g.z); h.a = hq(L.g.a); h.b = hq(L.g.b); h.out = hq(L.g.out);
                h.conv_w = L.g.conv_w.data(); h.A_log = L.g.A_log.data(); h.dt_bias = L.g.dt_bias.data();
                h.norm_w = L.g.norm_w.data();
            } else {
                h.q = hq(L.a.q); h.k = hq(L.a.k); h.v = hq(L.a.v); h.o = hq(L.a.o);
                h.q_norm = L.a.q_norm.data(); h.k_norm = L.a.k_norm.data();
            }
        }
        m->gt = qe_gtrunk_create(d, hq(m->embed), hq(m->lm_head), m->final_norm.data(), lh, dev);
        if (!m->gt) QE_FAIL("engine: the GPU trunk was not created (QE_TRUNK=host runs the trunk on the host)");
    }
    return 0;
}

}  // namespace

extern "C" {

QeModel *qe_load(const char *dir, int max_len) {
    if (!dir || max_len < 1) {
        fprintf(stderr, "qengine_b200: qe_load: bad arguments\n");
        return nullptr;
    }
    std::unique_ptr<QeModel> m(new QeModel());
    if (load_model(m.get(), dir, max_len)) return nullptr;
    return m.release();
}

void qe_free(QeModel *m) { delete m; }

void qe_reset(QeModel *m) {
    if (!m) return;
    if (m->gt && qe_gtrunk_reset(m->gt)) fprintf(stderr, "qengine_b200: qe_reset: GPU trunk reset failed\n");
    for (auto &L : m->layers) {
        if (L.linear) {
            std::fill(L.g.conv_state.begin(), L.g.conv_state.end(), 0.0f);
            std::fill(L.g.rec_state.begin(), L.g.rec_state.end(), 0.0f);
        } else {
            L.a.len = 0;
        }
    }
    m->pos = 0;
}

int qe_forward(QeModel *m, int token, float *logits) {
    if (!m || !logits) return -1;
    if (m->pos >= m->max_len) return -2;
    const Cfg &c = m->c;
    const int H = c.hidden;
    if (m->gt) {
        if (token < 0 || token >= c.vocab) return -1;
        if (qe_gtrunk_forward(m->gt, token, m->pos, logits)) return -1;
        m->pos++;
        return 0;
    }
    if (hq_row(m->embed, token, m->x.data())) return -1;
    for (auto &L : m->layers) {
        rmsnorm(m->t1.data(), m->x.data(), L.in_norm.data(), H, c.eps);
        const int rc = L.linear ? gdn_forward(m, L, m->t1.data(), m->t2.data())
                                : attn_forward(m, L, m->t1.data(), m->t2.data());
        if (rc) return rc;
        for (int i = 0; i < H; i++) m->h[(size_t)i] = m->x[(size_t)i] + m->t2[(size_t)i];
        rmsnorm(m->t1.data(), m->h.data(), L.post_norm.data(), H, c.eps);
        if (qe_moe_forward(L.moe, 1, m->t1.data(), m->t2.data())) return -1;
        for (int i = 0; i < H; i++) m->x[(size_t)i] = m->h[(size_t)i] + m->t2[(size_t)i];
    }
    rmsnorm(m->t1.data(), m->x.data(), m->final_norm.data(), H, c.eps);
    hq_matvec(m->lm_head, m->t1.data(), logits, m->gsum);
    m->pos++;
    return 0;
}

int qe_vocab(const QeModel *m) { return m ? m->c.vocab : -1; }
int qe_position(const QeModel *m) { return m ? m->pos : -1; }
int qe_max_len(const QeModel *m) { return m ? m->max_len : -1; }

void qe_trunk_rmsnorm(float *out, const float *x, const float *w, int n, float eps) { rmsnorm(out, x, w, n, eps); }
void qe_trunk_rope(float *x, int n_heads, int head_dim, int rot_dims, int pos, float theta) {
    rope(x, n_heads, head_dim, rot_dims, pos, theta);
}
void qe_trunk_conv_step(float *out, float *state, const float *x, const float *w, int C, int K) {
    conv_step(out, state, x, w, C, K);
}
void qe_trunk_l2norm(float *v, int n, float eps, float scale) { l2norm(v, n, eps, scale); }
void qe_trunk_gates(float *g, float *beta, const float *a, const float *b, const float *A_log, const float *dt_bias,
                    int Hv) {
    gates(g, beta, a, b, A_log, dt_bias, Hv);
}
void qe_trunk_recurrent_step(float *y, float *state, const float *q, const float *k, const float *v, const float *g,
                             const float *beta, int Hk, int Hv, int Dk, int Dv) {
    recurrent_step(y, state, q, k, v, g, beta, Hk, Hv, Dk, Dv);
}

}  // extern "C"
