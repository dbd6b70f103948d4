/* st_loader.cu: open one layer's MoE block from an MLX checkpoint directory (*.safetensors shards).
 *
 * The reference reads its checkpoints with a safetensors reader of its own (engine/src/io/k3_st.c:509-633:
 * every *.safetensors file of a directory, one flat JSON header per shard) and builds the block in load_moe
 * (engine/src/model.c:52-70): tensors <prefix>.switch_mlp.{gate,up,down}_proj, <prefix>.gate (router),
 * <prefix>.shared_expert.{gate,up,down}_proj and <prefix>.shared_expert_gate, each as .weight (U32 packed
 * codes), .scales and .biases (BF16), in the MLX affine layout (engine/include/qmat.h:3-11). Shapes follow
 * loader.c:16-41: cols = groups * group_size, bits = packed * 32 / cols; the routed experts are [E][rows][...].
 *
 * Here the shards are memory-mapped, the tensors are checked (dtype, shape, bounds) and handed to
 * qe_moe_create, which copies them (or this rank's expert slice) into HBM; the mappings are released before
 * returning. Host code only.
 */
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "qe_common.cuh"
#include "../../include/qe_moe.h"

namespace {

struct TensorInfo {
    std::string dtype;
    std::vector<int64_t> shape;
    int64_t begin = 0, end = 0;   /* byte offsets inside the shard's data section */
    int shard = -1;
};

struct Shard {
    std::string path;
    void *map = nullptr;
    size_t size = 0;
    size_t data0 = 0;             /* 8 + header length */
};

/* A parser for the rigid safetensors header: one object of name -> {dtype, shape, data_offsets}, plus an
 * optional "__metadata__" object of strings. Unknown members are skipped. */
struct Parser {
    const char *p, *end;
    bool ok = true;
    void ws() {
        while (p < end && (unsigned char)*p <= ' ') p++;
    }
    bool lit(char c) {
        ws();
        if (p < end && *p == c) {
            p++;
            return true;
        }
        return false;
    }
    bool str(std::string &out) {
        ws();
        if (p >= end || *p != '"') return ok = false;
        p++;
        out.clear();
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) return ok = false;
                const char c = *p;
                if (c == 'u') {   /* names are ASCII; keep the escape verbatim */
                    out += "\\u";
                } else {
                    out += c == 'n' ? '\n' : c == 't' ? '\t' : c;
                }
                p++;
                continue;
            }
            out += *p++;
        }
        if (p >= end) return ok = false;
        p++;
        return true;
    }
    bool i64(int64_t &v) {
        ws();
        bool neg = false;
        if (p < end && *p == '-') {
            neg = true;
            p++;
        }
        if (p >= end || *p < '0' || *p > '9') return ok = false;
        v = 0;
        while (p < end && *p >= '0' && *p <= '9') {
            if (v > (INT64_MAX - 9) / 10) return ok = false;
            v = v * 10 + (*p++ - '0');
        }
        if (neg) v = -v;
        return true;
    }
    bool skip() {   /* any JSON value */
        ws();
        if (p >= end) return ok = false;
        if (*p == '"') {
            std::string s;
            return str(s);
        }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            p++;
            if (lit(close)) return true;
            do {
                if (obj) {
                    std::string k;
                    if (!str(k) || !lit(':')) return ok = false;
                }
                if (!skip()) return false;
            } while (lit(','));
            if (lit(close)) return true;
            ok = false;
            return false;
        }
        while (p < end && *p != ',' && *p != '}' && *p != ']' && (unsigned char)*p > ' ') p++;
        return true;
    }
    bool tensor(TensorInfo &t) {
        if (!lit('{')) return ok = false;
        bool have_dtype = false, have_shape = false, have_off = false;
        if (lit('}')) return ok = false;
        do {
            std::string key;
            if (!str(key) || !lit(':')) return ok = false;
            if (key == "dtype") {
                if (!str(t.dtype)) return false;
                have_dtype = true;
            } else if (key == "shape") {
                if (!lit('[')) return ok = false;
                t.shape.clear();
                if (!lit(']')) {
                    do {
                        int64_t v;
                        if (!i64(v) || v < 0) return ok = false;
                        t.shape.push_back(v);
                    } while (lit(','));
                    if (!lit(']')) return ok = false;
                }
                have_shape = true;
            } else if (key == "data_offsets") {
                if (!lit('[') || !i64(t.begin) || !lit(',') || !i64(t.end) || !lit(']')) return ok = false;
                have_off = true;
            } else if (!skip()) {
                return false;
            }
        } while (lit(','));
        if (!lit('}')) return ok = false;
        return have_dtype && have_shape && have_off;
    }
};

int dtype_size(const std::string &d) {
    if (d == "U32" || d == "F32" || d == "I32") return 4;
    if (d == "BF16" || d == "F16" || d == "U16" || d == "I16") return 2;
    if (d == "U8" || d == "I8" || d == "BOOL") return 1;
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    return 0;
}

struct Checkpoint {
    std::vector<Shard> shards;
    std::map<std::string, TensorInfo> tensors;

    ~Checkpoint() {
        for (auto &s : shards)
            if (s.map) munmap(s.map, s.size);
    }

    int open_dir(const char *dir) {
        DIR *d = opendir(dir);
        if (!d) QE_FAIL("safetensors: cannot open directory %s", dir);
        std::vector<std::string> files;
        while (struct dirent *e = readdir(d)) {
            const std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
        }
        closedir(d);
        if (files.empty()) QE_FAIL("safetensors: no .safetensors files in %s", dir);
        std::sort(files.begin(), files.end());
        for (auto &f : files)
            if (add_shard(std::string(dir) + "/" + f)) return -1;
        return 0;
    }

    int add_shard(const std::string &path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) QE_FAIL("safetensors: cannot open %s", path.c_str());
        struct stat st;
        if (fstat(fd, &st) || st.st_size < 8) {
            ::close(fd);
            QE_FAIL("safetensors: %s is too short", path.c_str());
        }
        Shard sh;
        sh.path = path;
        sh.size = (size_t)st.st_size;
        sh.map = mmap(nullptr, sh.size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (sh.map == MAP_FAILED) {
            sh.map = nullptr;
            QE_FAIL("safetensors: cannot map %s", path.c_str());
        }
        const int idx = (int)shards.size();
        shards.push_back(sh);
        const unsigned char *b = (const unsigned char *)sh.map;
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | b[i];
        if (hlen > sh.size - 8) QE_FAIL("safetensors: %s: header length %llu beyond the file", path.c_str(),
                                        (unsigned long long)hlen);
        shards[idx].data0 = 8 + hlen;
        Parser ps{(const char *)b + 8, (const char *)b + 8 + hlen};
        if (!ps.lit('{')) QE_FAIL("safetensors: %s: header is not an object", path.c_str());
        if (!ps.lit('}')) {
            do {
                std::string name;
                if (!ps.str(name) || !ps.lit(':')) QE_FAIL("safetensors: %s: malformed header", path.c_str());
                if (name == "__metadata__") {
                    if (!ps.skip()) QE_FAIL("safetensors: %s: malformed metadata", path.c_str());
                    continue;
                }
                TensorInfo t;
                if (!ps.tensor(t)) QE_FAIL("safetensors: %s: malformed entry %s", path.c_str(), name.c_str());
                const int es = dtype_size(t.dtype);
                int64_t numel = 1;
                for (int64_t v : t.shape) numel *= v;
                if (es == 0 || t.begin < 0 || t.end < t.begin || (uint64_t)t.end > sh.size - shards[idx].data0 ||
                    t.end - t.begin != numel * es)
                    QE_FAIL("safetensors: %s: tensor %s has inconsistent dtype/shape/offsets", path.c_str(),
                            name.c_str());
                t.shard = idx;
                if (tensors.count(name)) QE_FAIL("safetensors: tensor %s appears twice", name.c_str());
                tensors[name] = t;
            } while (ps.lit(','));
            if (!ps.lit('}')) QE_FAIL("safetensors: %s: malformed header", path.c_str());
        }
        return 0;
    }

    const TensorInfo *find(const std::string &name) const {
        auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }
    const void *data(const TensorInfo &t) const {
        return (const char *)shards[t.shard].map + shards[t.shard].data0 + t.begin;
    }
};

/* One quantized tensor (loader.c:16-33): weight U32 [.., rows, packed], scales/biases BF16 [.., rows, groups]
 * with the same leading dimensions. n = product of the leading dimensions (experts). */
struct QView {
    QeQTensor t{};
    int64_t n = 0, rows = 0, packed = 0, groups = 0;
};

int qview(const Checkpoint &ck, const std::string &base, int ndim, QView &v) {
    const TensorInfo *w = ck.find(base + ".weight"), *s = ck.find(base + ".scales"), *b = ck.find(base + ".biases");
    if (!w || !s || !b) QE_FAIL("safetensors: missing %s.{weight,scales,biases}", base.c_str());
    if (w->dtype != "U32" || s->dtype != "BF16" || b->dtype != "BF16")
        QE_FAIL("safetensors: %s: expected U32 weight and BF16 scales/biases", base.c_str());
    if ((int)w->shape.size() != ndim || s->shape != b->shape || s->shape.size() != w->shape.size())
        QE_FAIL("safetensors: %s: unexpected rank", base.c_str());
    for (int i = 0; i + 1 < ndim; i++)
        if (w->shape[i] != s->shape[i]) QE_FAIL("safetensors: %s: weight and scales disagree", base.c_str());
    v.n = ndim == 3 ? w->shape[0] : 1;
    v.rows = w->shape[ndim - 2];
    v.packed = w->shape[ndim - 1];
    v.groups = s->shape[ndim - 1];
    v.t.w = (const uint32_t *)ck.data(*w);
    v.t.scales = (const uint16_t *)ck.data(*s);
    v.t.biases = (const uint16_t *)ck.data(*b);
    return 0;
}

}  // namespace

extern "C" {

int qe_safetensors_tensor_info(const char *dir, const char *name, char *dtype, int64_t *shape, int *ndim) {
    if (!dir || !name || !dtype || !shape || !ndim) QE_FAIL("safetensors: bad arguments");
    Checkpoint ck;
    if (ck.open_dir(dir)) return -1;
    const TensorInfo *t = ck.find(name);
    if (!t) QE_FAIL("safetensors: no tensor %s in %s", name, dir);
    if (t->shape.size() > 8) QE_FAIL("safetensors: %s has rank %zu > 8", name, t->shape.size());
    snprintf(dtype, 8, "%s", t->dtype.c_str());
    for (size_t i = 0; i < t->shape.size(); i++) shape[i] = t->shape[i];
    *ndim = (int)t->shape.size();
    return 0;
}

QeMoe *qe_moe_open_safetensors(const char *dir, const char *prefix, const QeMoeConfig *cfg_in) {
    if (!dir || !prefix || !cfg_in) {
        fprintf(stderr, "qengine_b200: open_safetensors: bad arguments\n");
        return nullptr;
    }
    Checkpoint ck;
    if (ck.open_dir(dir)) return nullptr;
    const std::string p = prefix;
    QView gate, up, down, sg, su, sd, rq, srq;
    if (qview(ck, p + ".switch_mlp.gate_proj", 3, gate) || qview(ck, p + ".switch_mlp.up_proj", 3, up) ||
        qview(ck, p + ".switch_mlp.down_proj", 3, down) || qview(ck, p + ".shared_expert.gate_proj", 2, sg) ||
        qview(ck, p + ".shared_expert.up_proj", 2, su) || qview(ck, p + ".shared_expert.down_proj", 2, sd) ||
        qview(ck, p + ".gate", 2, rq) || qview(ck, p + ".shared_expert_gate", 2, srq))
        return nullptr;
    QeMoeConfig c = *cfg_in;
    const int gs = c.group_size;
    if (gs != 32 && gs != 64 && gs != 128) {
        fprintf(stderr, "qengine_b200: open_safetensors: group_size %d not in {32, 64, 128}\n", gs);
        return nullptr;
    }
    /* shapes as loader.c:26 derives them: cols = groups * gs, bits = packed * 32 / cols */
    const int64_t hidden = gate.groups * gs, inter = down.groups * gs, sh_inter = sd.groups * gs;
    const int64_t bits = hidden ? gate.packed * 32 / hidden : 0, rbits = hidden ? rq.packed * 32 / hidden : 0;
    const bool shapes_ok =
        hidden > 0 && (bits == 4 || bits == 8) && gate.packed * 32 == bits * hidden && up.n == gate.n &&
        down.n == gate.n && up.rows == gate.rows && up.packed == gate.packed && gate.rows == inter &&
        down.rows == hidden && down.packed * 32 == bits * inter && sg.rows == sh_inter && su.rows == sh_inter &&
        sg.packed == gate.packed && su.packed == gate.packed && sd.rows == hidden && sd.packed * 32 == bits * sh_inter &&
        rq.rows == gate.n && (rbits == 4 || rbits == 8) && rq.packed * 32 == rbits * hidden && srq.rows == 1 &&
        srq.packed == rq.packed;
    if (!shapes_ok) {
        fprintf(stderr, "qengine_b200: open_safetensors: %s: tensor shapes do not form one MoE block\n", prefix);
        return nullptr;
    }
    auto check = [&](int given, int64_t found, const char *what) {
        if (given && given != found) {
            fprintf(stderr, "qengine_b200: open_safetensors: %s=%d given, checkpoint has %lld\n", what, given,
                    (long long)found);
            return false;
        }
        return true;
    };
    if (!check(c.hidden, hidden, "hidden") || !check(c.E, gate.n, "E") || !check(c.inter, inter, "inter") ||
        !check(c.sh_inter, sh_inter, "sh_inter") || !check(c.bits, bits, "bits"))
        return nullptr;
    c.hidden = (int)hidden;
    c.E = (int)gate.n;
    c.inter = (int)inter;
    c.sh_inter = (int)sh_inter;
    c.bits = (int)bits;
    c.router_mode = QE_ROUTER_QMAT;
    c.router_bits = (int)rbits;
    QeMoeWeights w = {};
    w.router_q = rq.t;
    w.sh_router_q = srq.t;
    w.gate = gate.t;
    w.up = up.t;
    w.down = down.t;
    w.sh_gate = sg.t;
    w.sh_up = su.t;
    w.sh_down = sd.t;
    return qe_moe_create(&c, &w);   /* copies into HBM; the mappings go away with ck */
}

}  // extern "C"
