/* ckpt.h: memory-mapped MLX safetensors checkpoints (every *.safetensors shard of a directory), shared by the
 * MoE-block loader (st_loader.cu) and the whole-model engine (engine.cu). Host code only, internal to
 * libqengine_b200.
 *
 * The reference reads its checkpoints with a reader of its own (engine/src/io/k3_st.c:509-633: every
 * *.safetensors file of a directory, one flat JSON header per shard). Here each shard is mapped read-only and
 * its header parsed into name -> (dtype, shape, byte range); tensors are handed out as pointers into the
 * mappings, which live as long as the Checkpoint.
 */
#ifndef QE_CKPT_H
#define QE_CKPT_H
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "qe_common.cuh"
#include "../../include/qe_moe.h"

namespace qe_ckpt {

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

inline int dtype_size(const std::string &d) {
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

inline int qview(const Checkpoint &ck, const std::string &base, int ndim, QView &v) {
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

}  // namespace qe_ckpt

#endif
