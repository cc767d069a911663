// safetensors.cpp - checkpoint loader: sharded safetensors -> resident
// quantized weights.
//
// Restates the parts of src/weights.zig that feed the quantized linears:
//   WeightMap.load (:258-352): model.safetensors.index.json's weight_map
//     names the shards; they are visited in first-appearance order and each
//     tensor is taken from its shard, a name seen twice is DuplicateTensor;
//   checkShardFile (:241-255): only a shard's header is read - a u64 LE
//     length n with 0 < n <= 256 MiB (else BadHeader), then n bytes of JSON;
//   parseHeaderJson (:72-121): a JSON object whose entries other than
//     "__metadata__" are objects with a "dtype" string (BF16, F32, U32, U8,
//     else UnsupportedDtype) and a "shape" array of integers (else
//     BadHeader); a "conv1d.weight" tensor must end in a unit dimension
//     (else UnsupportedLayout);
//   inferQuantSpec (:132-185) over every header of the checkpoint.
// Data are read straight from the shard at 8 + n + data_offsets[0] when a
// tensor is loaded; then data_offsets must span exactly the shape's bytes
// inside the file (else BadHeader - the reference meets that check in
// mlx_load_safetensors; parseHeaderJson itself does not look at offsets).
// Name sanitising and the vision-tower drop (weights.zig:188-202) are
// model-specific and not restated: names are kept as the file has them.
#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <climits>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "internal.h"

using qmm::set_error;

namespace {

// ---- a small JSON reader (objects keep their key order) --------------------

struct JValue {
    enum Kind { kNull, kBool, kInt, kFloat, kString, kArray, kObject } kind = kNull;
    bool b = false;
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;
    const JValue* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JParser {
  public:
    JParser(const char* p, size_t n) : p_(p), end_(p + n) {}
    bool parse(JValue* out) {
        if (!value(out, 0)) return false;
        ws();
        return p_ == end_;
    }

  private:
    const char* p_;
    const char* end_;
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if ((size_t)(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void put_utf8(std::string* s, uint32_t c) {
        if (c < 0x80) {
            s->push_back((char)c);
        } else if (c < 0x800) {
            s->push_back((char)(0xC0 | (c >> 6)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        } else if (c < 0x10000) {
            s->push_back((char)(0xE0 | (c >> 12)));
            s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        } else {
            s->push_back((char)(0xF0 | (c >> 18)));
            s->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
            s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        }
    }
    bool hex4(uint32_t* v) {
        if (end_ - p_ < 4) return false;
        *v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = *p_++;
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') *v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') *v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string* s) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_) {
            const char c = *p_++;
            if (c == '"') return true;
            if ((unsigned char)c < 0x20) return false;
            if (c != '\\') {
                s->push_back(c);
                continue;
            }
            if (p_ >= end_) return false;
            const char e = *p_++;
            switch (e) {
                case '"': s->push_back('"'); break;
                case '\\': s->push_back('\\'); break;
                case '/': s->push_back('/'); break;
                case 'b': s->push_back('\b'); break;
                case 'f': s->push_back('\f'); break;
                case 'n': s->push_back('\n'); break;
                case 'r': s->push_back('\r'); break;
                case 't': s->push_back('\t'); break;
                case 'u': {
                    uint32_t c1;
                    if (!hex4(&c1)) return false;
                    if (c1 >= 0xD800 && c1 < 0xDC00) {
                        uint32_t c2;
                        if (!lit("\\u") || !hex4(&c2) || c2 < 0xDC00 || c2 >= 0xE000) return false;
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    } else if (c1 >= 0xDC00 && c1 < 0xE000) {
                        return false;
                    }
                    put_utf8(s, c1);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    bool number(JValue* v) {
        const char* start = p_;
        if (p_ < end_ && *p_ == '-') ++p_;
        if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
        if (*p_ == '0') ++p_;
        else while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        bool frac = false;
        if (p_ < end_ && *p_ == '.') {
            frac = true;
            ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            frac = true;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        const std::string tok(start, p_);
        if (!frac) {
            errno = 0;
            char* e = nullptr;
            const long long x = std::strtoll(tok.c_str(), &e, 10);
            if (errno == 0 && e && *e == 0) {
                v->kind = JValue::kInt;
                v->i = x;
                return true;
            }
        }
        v->kind = JValue::kFloat;
        v->f = std::strtod(tok.c_str(), nullptr);
        return true;
    }
    bool value(JValue* v, int depth) {
        if (depth > 64) return false;
        ws();
        if (p_ >= end_) return false;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v->kind = JValue::kObject;
            ws();
            if (p_ < end_ && *p_ == '}') { ++p_; return true; }
            for (;;) {
                ws();
                std::string key;
                if (!string(&key)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                JValue child;
                if (!value(&child, depth + 1)) return false;
                v->obj.emplace_back(std::move(key), std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == '}') { ++p_; return true; }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v->kind = JValue::kArray;
            ws();
            if (p_ < end_ && *p_ == ']') { ++p_; return true; }
            for (;;) {
                JValue child;
                if (!value(&child, depth + 1)) return false;
                v->arr.push_back(std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == ']') { ++p_; return true; }
                return false;
            }
        }
        if (c == '"') {
            v->kind = JValue::kString;
            return string(&v->s);
        }
        if (lit("true")) { v->kind = JValue::kBool; v->b = true; return true; }
        if (lit("false")) { v->kind = JValue::kBool; v->b = false; return true; }
        if (lit("null")) { v->kind = JValue::kNull; return true; }
        return number(v);
    }
};

// ---- checkpoint ---------------------------------------------------------------

constexpr uint64_t kMaxHeader = 256ull * 1024 * 1024;   // weights.zig:250

struct Tensor {
    std::string name;
    int32_t dtype = 0;
    std::vector<int64_t> shape;
    int shard = 0;
    uint64_t begin = 0, end = 0;   // absolute file offsets of the data
};

int64_t dtype_bytes(int32_t dt) {
    switch (dt) {
        case QMM_DTYPE_BF16: return 2;
        case QMM_DTYPE_F32: return 4;
        case QMM_DTYPE_U32: return 4;
        default: return 1;
    }
}

bool read_at(int fd, void* dst, uint64_t n, uint64_t off) {
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n > 0) {
        const size_t chunk = (size_t)std::min<uint64_t>(n, 1ull << 30);
        const ssize_t r = ::pread(fd, d, chunk, (off_t)off);
        if (r <= 0) return false;
        d += r;
        n -= (uint64_t)r;
        off += (uint64_t)r;
    }
    return true;
}

// model_dir / file, as weights.zig joins them: shard names from the index
// are taken relative to the model directory.
std::string join(const std::string& dir, const std::string& f) {
    if (dir.empty()) return f;
    return dir.back() == '/' ? dir + f : dir + "/" + f;
}

}  // namespace

struct qmm_checkpoint {
    std::string dir;
    std::vector<std::string> shards;        // index order of first appearance
    std::vector<Tensor> tensors;            // shard order, then header order
    std::unordered_map<std::string, size_t> by_name;
    std::vector<qmm_tensor_info> infos;     // views for inferQuantSpec
    qmm_quant_spec spec{};
};

namespace {

// weights.zig:72-121 parseHeaderJson over one header; appends to `out`.
int parse_header_json(const char* json, size_t n, int shard, uint64_t data0, std::vector<Tensor>* out) {
    JValue root;
    JParser parser(json, n);
    if (!parser.parse(&root) || root.kind != JValue::kObject)
        return set_error(QMM_ERR_BAD_HEADER, "safetensors header is not a JSON object");
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JValue& o = kv.second;
        if (o.kind != JValue::kObject) return set_error(QMM_ERR_BAD_HEADER, "'%s' is not an object", kv.first.c_str());
        const JValue* dt = o.get("dtype");
        const JValue* sh = o.get("shape");
        if (!dt || !sh || dt->kind != JValue::kString || sh->kind != JValue::kArray)
            return set_error(QMM_ERR_BAD_HEADER, "'%s' lacks a dtype string or a shape array", kv.first.c_str());
        Tensor t;
        t.name = kv.first;
        if (dt->s == "BF16") t.dtype = QMM_DTYPE_BF16;
        else if (dt->s == "F32") t.dtype = QMM_DTYPE_F32;
        else if (dt->s == "U32") t.dtype = QMM_DTYPE_U32;
        else if (dt->s == "U8") t.dtype = QMM_DTYPE_U8;
        else return set_error(QMM_ERR_UNSUPPORTED_DTYPE, "'%s' has dtype %s", kv.first.c_str(), dt->s.c_str());
        for (const JValue& d : sh->arr) {
            if (d.kind != JValue::kInt) return set_error(QMM_ERR_BAD_HEADER, "'%s' shape is not integers", kv.first.c_str());
            t.shape.push_back(d.i);
        }
        if (t.name.find("conv1d.weight") != std::string::npos && (t.shape.empty() || t.shape.back() != 1))
            return set_error(QMM_ERR_UNSUPPORTED_LAYOUT, "'%s' must end in a unit dimension", t.name.c_str());
        // Data span, validated when the tensor is read.
        const JValue* offs = o.get("data_offsets");
        if (offs && offs->kind == JValue::kArray && offs->arr.size() == 2 && offs->arr[0].kind == JValue::kInt &&
            offs->arr[1].kind == JValue::kInt && offs->arr[0].i >= 0 && offs->arr[1].i >= offs->arr[0].i) {
            t.begin = data0 + (uint64_t)offs->arr[0].i;
            t.end = data0 + (uint64_t)offs->arr[1].i;
        } else {
            t.begin = t.end = 0;   // no usable span: reading it is BadHeader
        }
        t.shard = shard;
        out->push_back(std::move(t));
    }
    return QMM_OK;
}

// weights.zig:241-255 checkShardFile: the header only.
int check_shard(const std::string& path, int shard, std::vector<Tensor>* out) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(QMM_ERR_IO, "cannot open shard %s", path.c_str());
    uint8_t lenbuf[8];
    int rc = QMM_OK;
    if (!read_at(fd, lenbuf, 8, 0)) {
        rc = set_error(QMM_ERR_BAD_HEADER, "%s: shorter than the 8-byte header length", path.c_str());
    } else {
        uint64_t n = 0;
        for (int b = 7; b >= 0; --b) n = (n << 8) | lenbuf[b];
        if (n == 0 || n > kMaxHeader) {
            rc = set_error(QMM_ERR_BAD_HEADER, "%s: header length %llu outside (0, 256 MiB]", path.c_str(),
                           (unsigned long long)n);
        } else {
            std::vector<char> hdr(n);
            if (!read_at(fd, hdr.data(), n, 8)) rc = set_error(QMM_ERR_BAD_HEADER, "%s: truncated header", path.c_str());
            else rc = parse_header_json(hdr.data(), n, shard, 8 + n, out);
        }
    }
    ::close(fd);
    return rc;
}

bool read_file(const std::string& path, std::string* out) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return false;
    struct stat st;
    bool ok = ::fstat(fd, &st) == 0;
    if (ok) {
        out->resize((size_t)st.st_size);
        ok = read_at(fd, out->data(), (uint64_t)st.st_size, 0);
    }
    ::close(fd);
    return ok;
}

const Tensor* find(const qmm_checkpoint* c, const std::string& name) {
    auto it = c->by_name.find(name);
    return it == c->by_name.end() ? nullptr : &c->tensors[it->second];
}

// The tensor's byte count from its shape, or -1 (negative extent, overflow).
int64_t shape_bytes(const Tensor& t) {
    int64_t numel = 1;
    for (int64_t d : t.shape) {
        if (d < 0 || (d > 0 && numel > INT64_MAX / 8 / d)) return -1;
        numel *= d;
    }
    return numel * dtype_bytes(t.dtype);
}

int read_tensor(const qmm_checkpoint* c, const Tensor& t, void* dst) {
    const std::string path = join(c->dir, c->shards[t.shard]);
    const int64_t want = shape_bytes(t);
    if (want < 0 || t.end < t.begin || (uint64_t)want != t.end - t.begin || (want > 0 && t.begin == 0))
        return set_error(QMM_ERR_BAD_HEADER, "'%s': data_offsets do not span its %lld bytes", t.name.c_str(),
                         (long long)want);
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(QMM_ERR_IO, "cannot open shard %s", path.c_str());
    struct stat st;
    if (::fstat(fd, &st) != 0 || t.end > (uint64_t)st.st_size) {
        ::close(fd);
        return set_error(QMM_ERR_BAD_HEADER, "'%s' runs past the end of %s", t.name.c_str(), path.c_str());
    }
    const bool ok = read_at(fd, dst, t.end - t.begin, t.begin);
    ::close(fd);
    if (!ok) return set_error(QMM_ERR_IO, "short read of '%s' from %s", t.name.c_str(), path.c_str());
    return QMM_OK;
}

// "<prefix>.weight" (U32 [N, K*bits/32]) and "<prefix>.scales" (U8 [N, K/group])
// into host buffers, with (n, k) from the checkpoint's spec.
int read_linear(const qmm_checkpoint* c, const char* prefix, std::vector<uint8_t>* codes,
                std::vector<uint8_t>* scales, int64_t* n, int64_t* k) {
    if (!prefix) return set_error(QMM_ERR_BAD_ARGUMENT, "prefix is NULL");
    if (c->spec.mode == QMM_MODE_NONE) return set_error(QMM_ERR_NONSTANDARD_QUANT, "the checkpoint is not quantized");
    const std::string p(prefix);
    const Tensor* w = find(c, p + ".weight");
    const Tensor* s = find(c, p + ".scales");
    if (!w) return set_error(QMM_ERR_MISSING_TENSOR, "'%s.weight' is not in the checkpoint", prefix);
    if (!s) return set_error(QMM_ERR_MISSING_WEIGHT, "'%s.weight' has no scales", prefix);  // model.zig:226-228
    if (w->dtype != QMM_DTYPE_U32 || w->shape.size() != 2 || s->dtype != QMM_DTYPE_U8 || s->shape.size() != 2 ||
        w->shape[0] != s->shape[0])
        return set_error(QMM_ERR_BAD_SHAPE, "'%s': expected U32 [N, P] codes and U8 [N, G] scales", prefix);
    // Sizes first: the shape arithmetic below must not overflow on a hostile header.
    if (shape_bytes(*w) < 0 || shape_bytes(*s) < 0 || w->shape[1] > INT64_MAX / 32 || s->shape[1] > INT64_MAX / 32)
        return set_error(QMM_ERR_BAD_HEADER, "'%s': tensor sizes overflow", prefix);
    *n = w->shape[0];
    *k = w->shape[1] * 32 / c->spec.bits;
    if (s->shape[1] * c->spec.group_size != *k)
        return set_error(QMM_ERR_BAD_SHAPE, "'%s': %lld scale columns for k=%lld (group %d)", prefix,
                         (long long)s->shape[1], (long long)*k, c->spec.group_size);
    codes->resize((size_t)shape_bytes(*w));
    scales->resize((size_t)shape_bytes(*s));
    if (int rc = read_tensor(c, *w, codes->data())) return rc;
    return read_tensor(c, *s, scales->data());
}

}  // namespace

extern "C" int qmm_checkpoint_open(const char* model_dir, qmm_checkpoint** out) {
    if (!out || !model_dir) return set_error(QMM_ERR_BAD_ARGUMENT, "model_dir or out is NULL");
    *out = nullptr;
    auto c = std::make_unique<qmm_checkpoint>();
    c->dir = model_dir;
    std::string index;
    const std::string index_path = join(c->dir, "model.safetensors.index.json");
    if (!read_file(index_path, &index)) return set_error(QMM_ERR_IO, "cannot read %s", index_path.c_str());
    JValue root;
    JParser parser(index.data(), index.size());
    if (!parser.parse(&root) || root.kind != JValue::kObject)
        return set_error(QMM_ERR_BAD_INDEX_JSON, "%s is not a JSON object", index_path.c_str());
    const JValue* wm = root.get("weight_map");
    if (!wm || wm->kind != JValue::kObject)
        return set_error(QMM_ERR_BAD_INDEX_JSON, "%s has no weight_map object", index_path.c_str());
    for (const auto& kv : wm->obj) {
        if (kv.second.kind != JValue::kString)
            return set_error(QMM_ERR_BAD_INDEX_JSON, "weight_map['%s'] is not a file name", kv.first.c_str());
        bool seen = false;
        for (const auto& s : c->shards) seen = seen || s == kv.second.s;
        if (!seen) c->shards.push_back(kv.second.s);
    }
    for (size_t i = 0; i < c->shards.size(); ++i)
        if (int rc = check_shard(join(c->dir, c->shards[i]), (int)i, &c->tensors)) return rc;
    for (size_t i = 0; i < c->tensors.size(); ++i) {
        if (!c->by_name.emplace(c->tensors[i].name, i).second)
            return set_error(QMM_ERR_DUPLICATE_TENSOR, "'%s' appears twice", c->tensors[i].name.c_str());
    }
    c->infos.reserve(c->tensors.size());
    for (const Tensor& t : c->tensors)
        c->infos.push_back(qmm_tensor_info{t.name.c_str(), t.dtype, (int32_t)t.shape.size(), t.shape.data()});
    if (int rc = qmm_infer_quant_spec(c->infos.data(), (int64_t)c->infos.size(), &c->spec)) return rc;
    *out = c.release();
    return QMM_OK;
}

extern "C" int qmm_checkpoint_close(qmm_checkpoint* c) {
    delete c;
    return QMM_OK;
}

extern "C" int qmm_checkpoint_spec(const qmm_checkpoint* c, qmm_quant_spec* spec) {
    if (!c || !spec) return set_error(QMM_ERR_BAD_ARGUMENT, "checkpoint or spec is NULL");
    *spec = c->spec;
    return QMM_OK;
}

extern "C" int qmm_checkpoint_tensors(const qmm_checkpoint* c, const qmm_tensor_info** infos, int64_t* count) {
    if (!c || !infos || !count) return set_error(QMM_ERR_BAD_ARGUMENT, "null argument");
    *infos = c->infos.data();
    *count = (int64_t)c->infos.size();
    return QMM_OK;
}

extern "C" int qmm_checkpoint_read(const qmm_checkpoint* c, const char* name, void* dst, int64_t dst_bytes,
                                   int dst_kind) {
    if (!c || !name) return set_error(QMM_ERR_BAD_ARGUMENT, "null argument");
    const Tensor* t = find(c, name);
    if (!t) return set_error(QMM_ERR_MISSING_TENSOR, "'%s' is not in the checkpoint", name);
    if (!dst) return set_error(QMM_ERR_BAD_ARGUMENT, "dst is NULL");
    const int64_t nb = shape_bytes(*t);
    if (nb < 0) return set_error(QMM_ERR_BAD_HEADER, "'%s': tensor size overflows", name);
    const uint64_t n = (uint64_t)nb;
    if ((uint64_t)dst_bytes < n)
        return set_error(QMM_ERR_BAD_SHAPE, "'%s' needs %llu bytes, the buffer has %lld", name, (unsigned long long)n,
                         (long long)dst_bytes);
    if (dst_kind == QMM_SRC_HOST) return read_tensor(c, *t, dst);
    if (dst_kind != QMM_SRC_DEVICE) return set_error(QMM_ERR_BAD_ARGUMENT, "dst_kind %d", dst_kind);
    std::vector<uint8_t> host((size_t)n);
    if (int rc = read_tensor(c, *t, host.data())) return rc;
    QMM_CUDA_TRY(cudaMemcpy(dst, host.data(), (size_t)n, cudaMemcpyHostToDevice));
    return QMM_OK;
}

extern "C" int qmm_checkpoint_load_linear(const qmm_checkpoint* c, const char* prefix, void* stream,
                                          qmm_weight** out) {
    if (!c || !out) return set_error(QMM_ERR_BAD_ARGUMENT, "checkpoint or out is NULL");
    *out = nullptr;
    std::vector<uint8_t> codes, scales;
    int64_t n = 0, k = 0;
    if (int rc = read_linear(c, prefix, &codes, &scales, &n, &k)) return rc;
    return qmm_weight_create(codes.data(), scales.data(), n, k, 0, 0, c->spec, QMM_SRC_HOST, stream, out);
}

extern "C" int qmm_checkpoint_load_swiglu(const qmm_checkpoint* c, const char* gate_prefix, const char* up_prefix,
                                          void* stream, qmm_weight** out) {
    if (!c || !out) return set_error(QMM_ERR_BAD_ARGUMENT, "checkpoint or out is NULL");
    *out = nullptr;
    std::vector<uint8_t> gc, gs, uc, us;
    int64_t n = 0, k = 0, n2 = 0, k2 = 0;
    if (int rc = read_linear(c, gate_prefix, &gc, &gs, &n, &k)) return rc;
    if (int rc = read_linear(c, up_prefix, &uc, &us, &n2, &k2)) return rc;
    if (n != n2 || k != k2)
        return set_error(QMM_ERR_BAD_SHAPE, "gate [%lld, %lld] and up [%lld, %lld] differ", (long long)n, (long long)k,
                         (long long)n2, (long long)k2);
    return qmm_swiglu_weight_create(gc.data(), gs.data(), uc.data(), us.data(), n, k, 0, 0, c->spec, QMM_SRC_HOST,
                                    stream, out);
}
