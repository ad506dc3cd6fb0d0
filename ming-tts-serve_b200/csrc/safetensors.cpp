// safetensors.cpp — reads a model.safetensors checkpoint into a context
// (Model.load / Tensors.load, src/ming_model.zig:316-350,923-1005).
//
// File format (safetensors): an 8-byte little-endian header length n, n bytes
// of JSON mapping each tensor name to {"dtype", "shape", "data_offsets":
// [begin, end]} (offsets relative to the byte after the header; an optional
// "__metadata__" entry maps strings to strings), then the tensor bytes.
//
// The reference loads every tensor and casts all but int32 ones to the model
// dtype (bf16). Here only the tensors this library runs are read — names
// under model.model., stop_head, flowloss., linear_proj_audio, adaln_head,
// aggregator. and audio.decoder. — and handed to ming_cuda_load_tensor: BF16 and U32 (MLX
// packed quantized weights) as stored, F32 and F16 rounded to bf16 (nearest
// even), except rotary inv_freq buffers, which stay F32. Other dtypes and
// names are skipped.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/ming_cuda.h"

namespace ming {
namespace rt {
int fail(int code, const std::string& m);  // runtime.cu: the calling thread's last error
}  // namespace rt
}  // namespace ming

namespace {

// ---- a JSON reader for the header: objects, arrays, strings, numbers,
// true / false / null ----
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    double num = 0;
    long long inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const std::string& k) const {
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;
    int depth = 0;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool lit(const char* s) {
        const size_t n = std::strlen(s);
        if ((size_t)(end - p) < n || std::memcmp(p, s, n)) return false;
        p += n;
        return true;
    }
    static void utf8(std::string& o, unsigned cp) {
        if (cp < 0x80) o += (char)cp;
        else if (cp < 0x800) {
            o += (char)(0xC0 | (cp >> 6));
            o += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += (char)(0xE0 | (cp >> 12));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        } else {
            o += (char)(0xF0 | (cp >> 18));
            o += (char)(0x80 | ((cp >> 12) & 0x3F));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(unsigned& v) {
        if (end - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string& o) {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (true) {
            if (p >= end) return fail("unterminated string");
            const char c = *p++;
            if (c == '"') return true;
            if ((unsigned char)c < 0x20) return fail("control character in a string");
            if (c != '\\') {
                o += c;
                continue;
            }
            if (p >= end) return fail("unterminated escape");
            const char e = *p++;
            switch (e) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
                        unsigned lo;
                        if (!lit("\\u") || !hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(o, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
    }
    bool number(JVal& v) {
        const char* s = p;
        if (p < end && *p == '-') p++;
        bool digits = false, frac = false;
        while (p < end && *p >= '0' && *p <= '9') p++, digits = true;
        if (p < end && *p == '.') {
            frac = true;
            p++;
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            frac = true;
            p++;
            if (p < end && (*p == '+' || *p == '-')) p++;
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (!digits) return fail("bad number");
        const std::string t(s, p);
        v.kind = JVal::NUM;
        v.num = std::strtod(t.c_str(), nullptr);
        v.is_int = !frac && t.size() < 19;
        if (v.is_int) v.inum = std::strtoll(t.c_str(), nullptr, 10);
        return true;
    }
    bool value(JVal& v) {
        if (++depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end of header");
        bool ok = true;
        if (*p == '{') {
            v.kind = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') p++;
            else
                while (true) {
                    ws();
                    std::string k;
                    if (!string(k)) return false;
                    ws();
                    if (p >= end || *p != ':') return fail("expected ':'");
                    p++;
                    JVal x;
                    if (!value(x)) return false;
                    v.obj.emplace_back(std::move(k), std::move(x));
                    ws();
                    if (p < end && *p == ',') {
                        p++;
                        continue;
                    }
                    if (p < end && *p == '}') {
                        p++;
                        break;
                    }
                    return fail("expected ',' or '}'");
                }
        } else if (*p == '[') {
            v.kind = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') p++;
            else
                while (true) {
                    JVal x;
                    if (!value(x)) return false;
                    v.arr.push_back(std::move(x));
                    ws();
                    if (p < end && *p == ',') {
                        p++;
                        continue;
                    }
                    if (p < end && *p == ']') {
                        p++;
                        break;
                    }
                    return fail("expected ',' or ']'");
                }
        } else if (*p == '"') {
            v.kind = JVal::STR;
            ok = string(v.str);
        } else if (lit("true")) {
            v.kind = JVal::BOOL;
            v.inum = 1;
        } else if (lit("false")) {
            v.kind = JVal::BOOL;
        } else if (lit("null")) {
            v.kind = JVal::NUL;
        } else {
            ok = number(v);
        }
        depth--;
        return ok;
    }
};

// bf16 bit pattern of an f32 value, round to nearest even (NaN stays NaN)
uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    int e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu, u;
    if (e == 0x1F) u = s | 0x7F800000u | (m << 13);
    else if (e == 0) {
        if (!m) u = s;
        else {  // subnormal: normalise
            e = 1;
            while (!(m & 0x400u)) m <<= 1, e--;
            u = s | ((uint32_t)(e + 112) << 23) | ((m & 0x3FFu) << 13);
        }
    } else
        u = s | ((uint32_t)(e + 112) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

bool hot_path_name(const std::string& n) {
    static const char* pre[] = {"model.model.", "stop_head.", "flowloss.", "linear_proj_audio.", "adaln_head.", "aggregator.",
                                "audio.decoder."};
    for (const char* p : pre)
        if (n.compare(0, std::strlen(p), p) == 0) return true;
    return false;
}

bool ends_with(const std::string& s, const char* t) {
    const size_t n = std::strlen(t);
    return s.size() >= n && s.compare(s.size() - n, n, t) == 0;
}

struct Mapped {
    void* base = MAP_FAILED;
    size_t size = 0;
    int fd = -1;
    ~Mapped() {
        if (base != MAP_FAILED) munmap(base, size);
        if (fd >= 0) close(fd);
    }
};

int st_fail(int code, const std::string& m) { return ming::rt::fail(code, m); }

}  // namespace

extern "C" int ming_cuda_load_safetensors(ming_ctx* ctx, const char* path, int* n_loaded) {
    if (!path) return st_fail(MING_ERR_INVALID, "null path");
    std::string file = path;
    struct stat sb;
    if (stat(file.c_str(), &sb) == 0 && S_ISDIR(sb.st_mode)) file += "/model.safetensors";  // Model.load(model_dir)
    Mapped m;
    m.fd = open(file.c_str(), O_RDONLY);
    if (m.fd < 0) return st_fail(MING_ERR_INVALID, "cannot open " + file);
    if (fstat(m.fd, &sb) != 0) return st_fail(MING_ERR_INVALID, "cannot stat " + file);
    m.size = (size_t)sb.st_size;
    if (m.size < 8) return st_fail(MING_ERR_INVALID, file + ": too short for a safetensors header");
    m.base = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, m.fd, 0);
    if (m.base == MAP_FAILED) return st_fail(MING_ERR_INVALID, "cannot map " + file);
    const uint8_t* b = static_cast<const uint8_t*>(m.base);
    uint64_t hn = 0;
    for (int i = 0; i < 8; i++) hn |= (uint64_t)b[i] << (8 * i);
    if (hn > m.size - 8) return st_fail(MING_ERR_INVALID, file + ": header length past the end of the file");
    JParser jp{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hn)};
    JVal root;
    if (!jp.value(root)) return st_fail(MING_ERR_INVALID, file + ": bad header: " + jp.err);
    jp.ws();
    if (jp.p != jp.end) return st_fail(MING_ERR_INVALID, file + ": bad header: trailing bytes");
    if (root.kind != JVal::OBJ) return st_fail(MING_ERR_INVALID, file + ": header is not an object");
    const uint8_t* data = b + 8 + hn;
    const uint64_t dsize = m.size - 8 - hn;
    int loaded = 0;
    for (auto& kv : root.obj) {
        const std::string& name = kv.first;
        if (name == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
        if (t.kind != JVal::OBJ || !dt || dt->kind != JVal::STR || !sh || sh->kind != JVal::ARR || !off ||
            off->kind != JVal::ARR || off->arr.size() != 2)
            return st_fail(MING_ERR_INVALID, file + ": malformed entry " + name);
        std::vector<int64_t> shape;
        uint64_t count = 1;
        for (const JVal& d : sh->arr) {
            if (d.kind != JVal::NUM || !d.is_int || d.inum < 0) return st_fail(MING_ERR_INVALID, file + ": bad shape of " + name);
            shape.push_back(d.inum);
            if (d.inum && count > UINT64_MAX / (uint64_t)d.inum) return st_fail(MING_ERR_INVALID, file + ": shape overflow in " + name);
            count *= (uint64_t)d.inum;
        }
        if (shape.size() > 4) {
            if (hot_path_name(name)) return st_fail(MING_ERR_INVALID, file + ": more than 4 dimensions in " + name);
            continue;
        }
        for (const JVal& o : off->arr)
            if (o.kind != JVal::NUM || !o.is_int || o.inum < 0) return st_fail(MING_ERR_INVALID, file + ": bad offsets of " + name);
        const uint64_t o0 = (uint64_t)off->arr[0].inum, o1 = (uint64_t)off->arr[1].inum;
        size_t esz = 0;
        const std::string& d = dt->str;
        if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") esz = 2;
        else if (d == "F32" || d == "U32" || d == "I32") esz = 4;
        else if (d == "F64" || d == "I64" || d == "U64") esz = 8;
        else if (d == "U8" || d == "I8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") esz = 1;
        else return st_fail(MING_ERR_INVALID, file + ": unknown dtype " + d + " of " + name);
        if (o1 < o0 || o1 > dsize || o1 - o0 != count * esz)
            return st_fail(MING_ERR_INVALID, file + ": data offsets of " + name + " do not match its shape and dtype");
        if (!hot_path_name(name)) continue;
        const uint8_t* src = data + o0;
        const bool keep_f32 = ends_with(name, "inv_freq");
        int dtype = -1;
        std::vector<uint8_t> conv;
        if (d == "BF16") dtype = MING_DTYPE_BF16;
        else if (d == "U32") dtype = MING_DTYPE_U32;
        else if (d == "F32" && keep_f32) dtype = MING_DTYPE_F32;
        else if (d == "F32" || d == "F16") {
            dtype = MING_DTYPE_BF16;
            conv.resize(count * 2);
            uint16_t* o = reinterpret_cast<uint16_t*>(conv.data());
            for (uint64_t i = 0; i < count; i++) {
                float f;
                if (d == "F32") std::memcpy(&f, src + 4 * i, 4);
                else {
                    uint16_t h;
                    std::memcpy(&h, src + 2 * i, 2);
                    f = f16_to_f32(h);
                }
                o[i] = to_bf16(f);
            }
            src = conv.data();
        } else
            continue;  // integer tables and the like: not on the hot path
        loaded++;
        if (!ctx) continue;  // validation only
        const int rc = ming_cuda_load_tensor(ctx, name.c_str(), dtype, shape.data(), (int)shape.size(), src);
        if (rc) return st_fail(rc, name + ": " + std::string(ming_cuda_last_error()));
    }
    if (n_loaded) *n_loaded = loaded;
    return MING_OK;
}
