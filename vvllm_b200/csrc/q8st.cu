// q8st.cu -- safetensors files on either side of the quantize step (host code).
//
// vvllm loads a checkpoint by mmapping a safetensors file (src/safetensors/safetensors.cc:
// 43-83: 8-byte little-endian header length, JSON header of {name: {dtype, shape,
// data_offsets}}, then the data), widening BF16 to fp32 on the host (:101-117) and quantizing
// every projection on the host at load (src/model/qwen2/model.cc:27-38).  This file gives
//   * a reader with the same layout rules (mmap, header parsed once, pointers into the map), and
//   * a converter that writes a quantized safetensors file: each projection "<name>" becomes
//     "<name>.q8" (I8 [N, K]) and "<name>.q8_scales" (F32 [N]), quantized on the GPU with the
//     bit-exact quantize kernels (fp32 or bf16 source); all other tensors are copied byte for
//     byte.  Loading such a file needs no quantize step at all.
// The header is parsed by a small JSON reader of its own (objects, arrays, strings, integers,
// true/false/null: what safetensors headers contain).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "b200q8.h"
#include "kernels.h"

namespace {

using b200q8::cuda_fail;
using b200q8::fail;

// ------------------------------------------------------------------------------------ JSON
struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    bool b = false;
    bool num_int = false;     // the number is a non-negative integer that fits in 64 bits
    unsigned long long u = 0;
    std::string s;            // string value, or a number's text
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* key) const
    {
        for (auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JParser {
public:
    JParser(const char* p, size_t n) : p_(p), e_(p + n) {}
    bool parse(JVal* out)
    {
        if (!value(out, 0)) return false;
        ws();
        return p_ == e_;
    }

private:
    const char* p_;
    const char* e_;

    void ws()
    {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
    }
    bool lit(const char* w)
    {
        const size_t n = strlen(w);
        if ((size_t)(e_ - p_) < n || memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void put_utf8(std::string* s, unsigned cp)
    {
        if (cp < 0x80) {
            s->push_back((char)cp);
        } else if (cp < 0x800) {
            s->push_back((char)(0xC0 | (cp >> 6)));
            s->push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            s->push_back((char)(0xE0 | (cp >> 12)));
            s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            s->push_back((char)(0xF0 | (cp >> 18)));
            s->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    // The rest of a UTF-8 sequence whose lead byte is c (already consumed): well-formed, shortest
    // form, no surrogates, at most U+10FFFF.
    bool utf8_tail(unsigned char c, std::string* out)
    {
        int n;
        unsigned cp;
        if (c >= 0xC2 && c <= 0xDF) { n = 1; cp = c & 0x1F; }
        else if (c >= 0xE0 && c <= 0xEF) { n = 2; cp = c & 0x0F; }
        else if (c >= 0xF0 && c <= 0xF4) { n = 3; cp = c & 0x07; }
        else return false;
        if (e_ - p_ < n) return false;
        out->push_back((char)c);
        for (int i = 0; i < n; i++) {
            const unsigned char t = (unsigned char)*p_++;
            if ((t & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (t & 0x3F);
            out->push_back((char)t);
        }
        if ((n == 2 && cp < 0x800) || (n == 3 && cp < 0x10000) || cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000))
            return false;
        return true;
    }
    bool hex4(unsigned* v)
    {
        if (e_ - p_ < 4) return false;
        unsigned r = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p_++;
            r <<= 4;
            if (c >= '0' && c <= '9') r |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') r |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') r |= (unsigned)(c - 'A' + 10);
            else return false;
        }
        *v = r;
        return true;
    }
    bool str(std::string* out)
    {
        if (p_ >= e_ || *p_ != '"') return false;
        p_++;
        out->clear();
        while (p_ < e_ && *p_ != '"') {
            const unsigned char c = (unsigned char)*p_++;
            if (c < 0x20) return false;
            if (c >= 0x80) {  // a UTF-8 sequence: JSON text must be valid UTF-8
                if (!utf8_tail(c, out)) return false;
                continue;
            }
            if (c != '\\') {
                out->push_back((char)c);
                continue;
            }
            if (p_ >= e_) return false;
            const char x = *p_++;
            switch (x) {
                case '"': out->push_back('"'); break;
                case '\\': out->push_back('\\'); break;
                case '/': out->push_back('/'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'n': out->push_back('\n'); break;
                case 'r': out->push_back('\r'); break;
                case 't': out->push_back('\t'); break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
                        unsigned lo;
                        if (!lit("\\u") || !hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    put_utf8(out, cp);
                    break;
                }
                default: return false;
            }
        }
        if (p_ >= e_) return false;
        p_++;
        return true;
    }
    bool num(JVal* v)
    {
        const char* b = p_;
        if (p_ < e_ && *p_ == '-') p_++;
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        bool integral = true;
        if (p_ < e_ && *p_ == '.') {
            integral = false;
            p_++;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            p_++;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) p_++;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') p_++;
        }
        v->kind = JVal::kNum;
        v->s.assign(b, p_);
        v->num_int = false;
        if (integral && *b != '-' && p_ - b <= 20) {
            unsigned long long u = 0;
            bool ok = true;
            for (const char* c = b; c < p_; c++) {
                const unsigned d = (unsigned)(*c - '0');
                if (u > (~0ull - d) / 10) {
                    ok = false;
                    break;
                }
                u = u * 10 + d;
            }
            v->num_int = ok;
            v->u = u;
        }
        return true;
    }
    bool value(JVal* v, int depth)
    {
        if (depth > 64) return false;
        ws();
        if (p_ >= e_) return false;
        const char c = *p_;
        if (c == '{') {
            p_++;
            v->kind = JVal::kObj;
            ws();
            if (p_ < e_ && *p_ == '}') {
                p_++;
                return true;
            }
            for (;;) {
                ws();
                std::pair<std::string, JVal> kv;
                if (!str(&kv.first)) return false;
                ws();
                if (p_ >= e_ || *p_ != ':') return false;
                p_++;
                if (!value(&kv.second, depth + 1)) return false;
                v->obj.push_back(std::move(kv));
                ws();
                if (p_ < e_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < e_ && *p_ == '}') {
                    p_++;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            p_++;
            v->kind = JVal::kArr;
            ws();
            if (p_ < e_ && *p_ == ']') {
                p_++;
                return true;
            }
            for (;;) {
                JVal x;
                if (!value(&x, depth + 1)) return false;
                v->arr.push_back(std::move(x));
                ws();
                if (p_ < e_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < e_ && *p_ == ']') {
                    p_++;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v->kind = JVal::kStr;
            return str(&v->s);
        }
        if (lit("true")) {
            v->kind = JVal::kBool;
            v->b = true;
            return true;
        }
        if (lit("false")) {
            v->kind = JVal::kBool;
            return true;
        }
        if (lit("null")) {
            v->kind = JVal::kNull;
            return true;
        }
        return num(v);
    }
};

void json_str(std::string* out, const std::string& s)
{
    out->push_back('"');
    for (unsigned char c : s) {
        if (c == '"' || c == '\\') {
            out->push_back('\\');
            out->push_back((char)c);
        } else if (c < 0x20) {
            char buf[8];
            snprintf(buf, sizeof buf, "\\u%04x", c);
            out->append(buf);
        } else {
            out->push_back((char)c);
        }
    }
    out->push_back('"');
}

// --------------------------------------------------------------------------- dtypes
struct DtypeName {
    const char* name;
    int code;
    size_t bytes;
};
const DtypeName kDtypes[] = {
    {"F32", B200Q8_ST_F32, 4},   {"F16", B200Q8_ST_F16, 2},   {"BF16", B200Q8_ST_BF16, 2},
    {"I8", B200Q8_ST_I8, 1},     {"U8", B200Q8_ST_OTHER, 1},  {"BOOL", B200Q8_ST_OTHER, 1},
    {"I16", B200Q8_ST_OTHER, 2}, {"U16", B200Q8_ST_OTHER, 2}, {"I32", B200Q8_ST_OTHER, 4},
    {"U32", B200Q8_ST_OTHER, 4}, {"F64", B200Q8_ST_OTHER, 8}, {"I64", B200Q8_ST_OTHER, 8},
    {"U64", B200Q8_ST_OTHER, 8}, {"F8_E4M3", B200Q8_ST_OTHER, 1}, {"F8_E5M2", B200Q8_ST_OTHER, 1},
};
const DtypeName* find_dtype(const std::string& s)
{
    for (auto& d : kDtypes)
        if (s == d.name) return &d;
    return nullptr;
}

}  // namespace

// ------------------------------------------------------------------------------- reader
struct b200q8_st {
    int fd = -1;
    void* map = MAP_FAILED;
    size_t size = 0;
    const uint8_t* data = nullptr;  // start of the tensor data
    size_t data_size = 0;
    struct Entry {
        std::string name;
        std::string dtype;  // as written in the file
        int code = B200Q8_ST_OTHER;
        std::vector<size_t> shape;
        size_t begin = 0, end = 0;
    };
    std::vector<Entry> entries;  // in file-data order
    std::unordered_map<std::string, size_t> index;
    std::vector<std::pair<std::string, std::string>> metadata;  // "__metadata__" (string values)
    ~b200q8_st()
    {
        if (map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
};

namespace {

int parse_header(b200q8_st* f, const char* path)
{
    if (f->size < 8) return fail(B200Q8_ERR_INVALID, "safetensors %s: file shorter than its 8-byte header length", path);
    uint64_t hlen = 0;
    memcpy(&hlen, f->map, 8);  // little-endian, as every platform vvllm targets
    if (hlen > f->size - 8 || hlen > ((uint64_t)100 << 20))
        return fail(B200Q8_ERR_INVALID, "safetensors %s: header length %llu exceeds the file / 100 MB", path,
                    (unsigned long long)hlen);
    const char* h = static_cast<const char*>(f->map) + 8;
    JVal root;
    JParser jp(h, (size_t)hlen);
    if (!jp.parse(&root) || root.kind != JVal::kObj)
        return fail(B200Q8_ERR_INVALID, "safetensors %s: header is not a JSON object", path);
    f->data = static_cast<const uint8_t*>(f->map) + 8 + hlen;
    f->data_size = f->size - 8 - (size_t)hlen;
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != JVal::kObj)
                return fail(B200Q8_ERR_INVALID, "safetensors %s: __metadata__ is not an object", path);
            for (auto& m : kv.second.obj) {
                if (m.second.kind != JVal::kStr)
                    return fail(B200Q8_ERR_INVALID, "safetensors %s: __metadata__ value is not a string", path);
                f->metadata.emplace_back(m.first, m.second.s);
            }
            continue;
        }
        const JVal& t = kv.second;
        const JVal* dt = t.kind == JVal::kObj ? t.get("dtype") : nullptr;
        const JVal* sh = t.kind == JVal::kObj ? t.get("shape") : nullptr;
        const JVal* off = t.kind == JVal::kObj ? t.get("data_offsets") : nullptr;
        if (!dt || dt->kind != JVal::kStr || !sh || sh->kind != JVal::kArr || !off || off->kind != JVal::kArr ||
            off->arr.size() != 2 || !off->arr[0].num_int || !off->arr[1].num_int)
            return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' lacks dtype / shape / data_offsets", path,
                        kv.first.c_str());
        b200q8_st::Entry e;
        e.name = kv.first;
        e.dtype = dt->s;
        const DtypeName* d = find_dtype(dt->s);
        if (!d) return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' has unknown dtype '%s'", path,
                            kv.first.c_str(), dt->s.c_str());
        e.code = d->code;
        size_t count = 1;
        for (auto& x : sh->arr) {
            if (!x.num_int) return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' has a bad shape", path,
                                        kv.first.c_str());
            if (x.u && count > SIZE_MAX / x.u)
                return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' size overflows", path, kv.first.c_str());
            count *= (size_t)x.u;
            e.shape.push_back((size_t)x.u);
        }
        e.begin = (size_t)off->arr[0].u;
        e.end = (size_t)off->arr[1].u;
        if (e.begin > e.end || e.end > f->data_size)
            return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' data_offsets [%zu, %zu) outside the %zu data bytes",
                        path, kv.first.c_str(), e.begin, e.end, f->data_size);
        if (count > SIZE_MAX / d->bytes || e.end - e.begin != count * d->bytes)
            return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' holds %zu bytes, its shape needs %zu", path,
                        kv.first.c_str(), e.end - e.begin, count * d->bytes);
        f->entries.push_back(std::move(e));
    }
    std::sort(f->entries.begin(), f->entries.end(),
              [](const b200q8_st::Entry& a, const b200q8_st::Entry& b) { return a.begin < b.begin; });
    for (size_t i = 0; i < f->entries.size(); i++) {
        if (i && f->entries[i].begin < f->entries[i - 1].end)
            return fail(B200Q8_ERR_INVALID, "safetensors %s: tensors '%s' and '%s' overlap", path,
                        f->entries[i - 1].name.c_str(), f->entries[i].name.c_str());
        if (!f->index.emplace(f->entries[i].name, i).second)
            return fail(B200Q8_ERR_INVALID, "safetensors %s: tensor '%s' appears twice", path,
                        f->entries[i].name.c_str());
    }
    return B200Q8_OK;
}

// Projections quantized by the converter: the linear weights vvllm quantizes at load
// (model.cc:40-80: self_attn.{q,k,v,o}_proj and mlp.{gate,up,down}_proj), recognised by the
// "_proj.weight" suffix; with B200Q8_ST_LM_HEAD also the output head.
bool is_projection(const b200q8_st::Entry& e)
{
    static const char kSuffix[] = "_proj.weight";
    const size_t n = sizeof(kSuffix) - 1;
    return e.shape.size() == 2 && (e.code == B200Q8_ST_F32 || e.code == B200Q8_ST_BF16) && e.name.size() > n &&
           e.name.compare(e.name.size() - n, n, kSuffix) == 0;
}

struct OutTensor {
    std::string name, dtype;
    std::vector<size_t> shape;
    size_t bytes = 0;
    int src = -1;       // index of the source entry
    int part = 0;       // 0: copied source bytes; 1: quantized data; 2: scales
};

int write_all(FILE* fp, const void* p, size_t n, const char* path)
{
    if (n && fwrite(p, 1, n, fp) != n) return fail(B200Q8_ERR_IO, "safetensors %s: write failed", path);
    return B200Q8_OK;
}

}  // namespace

extern "C" {

int b200q8_st_open(const char* path, b200q8_st** out)
{
    if (!path || !out) return fail(B200Q8_ERR_INVALID, "st_open: null argument");
    *out = nullptr;
    std::unique_ptr<b200q8_st> f(new b200q8_st());
    f->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (f->fd < 0) return fail(B200Q8_ERR_IO, "safetensors %s: cannot open", path);
    struct stat st;
    if (fstat(f->fd, &st) != 0) return fail(B200Q8_ERR_IO, "safetensors %s: cannot stat", path);
    f->size = (size_t)st.st_size;
    if (f->size == 0) return fail(B200Q8_ERR_INVALID, "safetensors %s: empty file", path);
    f->map = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
    if (f->map == MAP_FAILED) return fail(B200Q8_ERR_IO, "safetensors %s: mmap failed", path);
    const int st2 = parse_header(f.get(), path);
    if (st2) return st2;
    *out = f.release();
    return B200Q8_OK;
}

int b200q8_st_close(b200q8_st* f)
{
    delete f;
    return B200Q8_OK;
}

int b200q8_st_count(const b200q8_st* f, size_t* n)
{
    if (!f || !n) return fail(B200Q8_ERR_INVALID, "st_count: null argument");
    *n = f->entries.size();
    return B200Q8_OK;
}

int b200q8_st_info(const b200q8_st* f, size_t i, const char** name, int* dtype, size_t* ndim, const size_t** shape,
                   const void** data, size_t* nbytes)
{
    if (!f) return fail(B200Q8_ERR_INVALID, "st_info: null file");
    if (i >= f->entries.size()) return fail(B200Q8_ERR_INVALID, "st_info: index %zu of %zu", i, f->entries.size());
    const auto& e = f->entries[i];
    if (name) *name = e.name.c_str();
    if (dtype) *dtype = e.code;
    if (ndim) *ndim = e.shape.size();
    if (shape) *shape = e.shape.data();
    if (data) *data = f->data + e.begin;
    if (nbytes) *nbytes = e.end - e.begin;
    return B200Q8_OK;
}

int b200q8_st_find(const b200q8_st* f, const char* name, size_t* i)
{
    if (!f || !name || !i) return fail(B200Q8_ERR_INVALID, "st_find: null argument");
    auto it = f->index.find(name);
    if (it == f->index.end()) return fail(B200Q8_ERR_NOT_FOUND, "st_find: no tensor '%s'", name);
    *i = it->second;
    return B200Q8_OK;
}

int b200q8_st_quantized(const b200q8_st* f, const char* name, size_t* N, size_t* K, const int8_t** q,
                        const float** scales)
{
    if (!f || !name) return fail(B200Q8_ERR_INVALID, "st_quantized: null argument");
    const std::string base(name);
    auto iq = f->index.find(base + ".q8");
    auto is = f->index.find(base + ".q8_scales");
    if (iq == f->index.end() || is == f->index.end())
        return fail(B200Q8_ERR_NOT_FOUND, "st_quantized: no quantized tensor '%s'", name);
    const auto& eq = f->entries[iq->second];
    const auto& es = f->entries[is->second];
    if (eq.code != B200Q8_ST_I8 || eq.shape.size() != 2 || es.code != B200Q8_ST_F32 || es.shape.size() != 1 ||
        es.shape[0] != eq.shape[0])
        return fail(B200Q8_ERR_INVALID, "st_quantized: '%s' is not an I8 [N, K] + F32 [N] pair", name);
    if (N) *N = eq.shape[0];
    if (K) *K = eq.shape[1];
    if (q) *q = reinterpret_cast<const int8_t*>(f->data + eq.begin);
    if (scales) *scales = reinterpret_cast<const float*>(f->data + es.begin);
    return B200Q8_OK;
}

int b200q8_st_quantize(const char* src_path, const char* dst_path, int device, unsigned int flags)
{
    if (!src_path || !dst_path) return fail(B200Q8_ERR_INVALID, "st_quantize: null path");
    b200q8_st* raw = nullptr;
    int st = b200q8_st_open(src_path, &raw);
    if (st) return st;
    std::unique_ptr<b200q8_st> src(raw);
    // Output tensors, in source-data order.
    const bool lm_head = (flags & B200Q8_ST_LM_HEAD) != 0;
    const bool has_lm_head = src->index.count("lm_head.weight") != 0;
    std::vector<OutTensor> outs;
    size_t max_src = 0, max_rows = 0, max_q = 0;
    for (size_t i = 0; i < src->entries.size(); i++) {
        const auto& e = src->entries[i];
        const bool proj = is_projection(e);
        const bool head_q = lm_head && e.shape.size() == 2 && (e.code == B200Q8_ST_F32 || e.code == B200Q8_ST_BF16) &&
                            (e.name == "lm_head.weight" || (!has_lm_head && e.name == "model.embed_tokens.weight"));
        // A tied head (embed_tokens) keeps its source tensor for the embedding lookup.
        const bool keep = !(proj || (head_q && e.name == "lm_head.weight"));
        if (keep) {
            OutTensor o;
            o.name = e.name;
            o.dtype = e.dtype;
            o.shape = e.shape;
            o.bytes = e.end - e.begin;
            o.src = (int)i;
            outs.push_back(o);
        }
        if (proj || head_q) {
            const size_t N = e.shape[0], K = e.shape[1];
            OutTensor q, s;
            q.name = e.name + ".q8";
            q.dtype = "I8";
            q.shape = {N, K};
            q.bytes = N * K;
            q.src = (int)i;
            q.part = 1;
            s.name = e.name + ".q8_scales";
            s.dtype = "F32";
            s.shape = {N};
            s.bytes = N * sizeof(float);
            s.src = (int)i;
            s.part = 2;
            if (src->index.count(q.name) || src->index.count(s.name))
                return fail(B200Q8_ERR_INVALID, "st_quantize: %s already holds '%s'", src_path, q.name.c_str());
            outs.push_back(q);
            outs.push_back(s);
            max_src = std::max(max_src, e.end - e.begin);
            max_rows = std::max(max_rows, N);
            max_q = std::max(max_q, N * K);
        }
    }
    // Header: metadata first (the source's, plus the format note), then the tensors.
    std::string h = "{\"__metadata__\":{";
    bool first = true;
    for (auto& m : src->metadata) {
        if (m.first == "b200q8") continue;
        if (!first) h += ",";
        json_str(&h, m.first);
        h += ":";
        json_str(&h, m.second);
        first = false;
    }
    if (!first) h += ",";
    h += "\"b200q8\":\"per-channel absmax int8 (vvllm quantize_per_channel): <name>.q8 I8 [N,K], "
         "<name>.q8_scales F32 [N]\"}";
    size_t off = 0;
    for (auto& o : outs) {
        h += ",";
        json_str(&h, o.name);
        h += ":{\"dtype\":";
        json_str(&h, o.dtype);
        h += ",\"shape\":[";
        for (size_t j = 0; j < o.shape.size(); j++) h += (j ? "," : "") + std::to_string(o.shape[j]);
        h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + o.bytes) + "]}";
        off += o.bytes;
    }
    h += "}";
    while ((8 + h.size()) % 8) h += " ";  // data starts 8-byte aligned
    // Device buffers for the largest projection.
    int prev = 0;
    cudaError_t ce = cudaGetDevice(&prev);
    if (ce != cudaSuccess) return cuda_fail(ce, "st_quantize: cudaGetDevice");
    if ((ce = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(ce, "st_quantize: cudaSetDevice");
    struct Dev {
        void* p = nullptr;
        ~Dev() { if (p) cudaFree(p); }
    } d_src, d_q, d_s;
    struct Host {
        void* p = nullptr;
        ~Host() { if (p) cudaFreeHost(p); }
    } h_q, h_s;
    cudaStream_t stream = nullptr;
    struct StreamGuard {
        cudaStream_t* s;
        int dev;
        ~StreamGuard()
        {
            if (*s) cudaStreamDestroy(*s);
            cudaSetDevice(dev);
        }
    } sg{&stream, prev};
    if (max_q &&
        ((ce = cudaMalloc(&d_src.p, max_src)) != cudaSuccess || (ce = cudaMalloc(&d_q.p, max_q)) != cudaSuccess ||
         (ce = cudaMalloc(&d_s.p, max_rows * sizeof(float))) != cudaSuccess ||
         (ce = cudaMallocHost(&h_q.p, max_q)) != cudaSuccess ||
         (ce = cudaMallocHost(&h_s.p, max_rows * sizeof(float))) != cudaSuccess ||
         (ce = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking)) != cudaSuccess)) {
        cudaGetLastError();
        return fail(B200Q8_ERR_ALLOC, "st_quantize: device / pinned buffers (%zu + %zu bytes): %s", max_src, max_q,
                    cudaGetErrorString(ce));
    }
    FILE* fp = fopen(dst_path, "wb");
    if (!fp) return fail(B200Q8_ERR_IO, "st_quantize: cannot create %s", dst_path);
    struct FileGuard {  // an incomplete output file is removed
        FILE* fp;
        const char* path;
        ~FileGuard()
        {
            if (fp) {
                fclose(fp);
                unlink(path);
            }
        }
    } fg{fp, dst_path};
    const uint64_t hlen = h.size();
    if ((st = write_all(fp, &hlen, 8, dst_path)) || (st = write_all(fp, h.data(), h.size(), dst_path))) return st;
    for (auto& o : outs) {
        const auto& e = src->entries[(size_t)o.src];
        const uint8_t* bytes = src->data + e.begin;
        if (o.part == 0) {
            if ((st = write_all(fp, bytes, o.bytes, dst_path))) return st;
        } else if (o.part == 1) {  // quantize now; the scales follow as the next output tensor
            const size_t N = e.shape[0], K = e.shape[1];
            if ((ce = cudaMemcpyAsync(d_src.p, bytes, e.end - e.begin, cudaMemcpyHostToDevice, stream)) != cudaSuccess)
                return cuda_fail(ce, "st_quantize: upload");
            st = e.code == B200Q8_ST_BF16
                     ? b200q8_quantize_per_channel_bf16(static_cast<const uint16_t*>(d_src.p), N, K,
                                                        static_cast<int8_t*>(d_q.p), static_cast<float*>(d_s.p),
                                                        stream)
                     : b200q8_quantize_per_channel(static_cast<const float*>(d_src.p), N, K,
                                                   static_cast<int8_t*>(d_q.p), static_cast<float*>(d_s.p), stream);
            if (st) return st;
            if ((ce = cudaMemcpyAsync(h_q.p, d_q.p, N * K, cudaMemcpyDeviceToHost, stream)) != cudaSuccess ||
                (ce = cudaMemcpyAsync(h_s.p, d_s.p, N * sizeof(float), cudaMemcpyDeviceToHost, stream)) !=
                    cudaSuccess ||
                (ce = cudaStreamSynchronize(stream)) != cudaSuccess)
                return cuda_fail(ce, "st_quantize: download");
            if ((st = write_all(fp, h_q.p, N * K, dst_path))) return st;
        } else {
            if ((st = write_all(fp, h_s.p, o.bytes, dst_path))) return st;
        }
    }
    fg.fp = nullptr;
    if (fclose(fp) != 0) {
        unlink(dst_path);
        return fail(B200Q8_ERR_IO, "st_quantize: closing %s failed", dst_path);
    }
    return B200Q8_OK;
}

}  // extern "C"
