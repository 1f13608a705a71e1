// pox_file.cpp -- the .pox container on the host: read-only mmap, header and section bounds, the JSON
// tensor index and model configuration, zero-copy payload slices, SHA-256 integrity, tensor-parallel
// shards of INT4 payloads and the model loader that uploads a whole .pox model to the GPU once.
//
// Reference: crates/paraoxidizer-format/src/pox.rs (PoxHeader :23-113, PoxFile::open / from_bytes /
// from_mmap :171-310, get_{tensor,scale,outlier}_data :311-353, verify_integrity :356-383, the writer's
// layout :397-606) and crates/paraoxidizer-core/src/tensor.rs:116-128 (TensorMeta). The layout is
// fixed by the format: a 128-byte little-endian header, JSON sections (serde_json) and 64-byte aligned
// payloads addressed by absolute offsets.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/pox_cuda.h"
#include "api_internal.h"

namespace {

using pox::set_error;

// ---------------------------------------------------------------------------------------------
// SHA-256 (FIPS 180-4)
// ---------------------------------------------------------------------------------------------
struct Sha256 {
    uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                     0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    uint8_t buf[64];
    size_t fill = 0;
    uint64_t total = 0;

    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

    void block(const uint8_t* p) {
        static const uint32_t k[64] = {
            0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
            0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
            0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
            0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
            0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
            0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
            0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
            0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
        uint32_t w[64];
        for (int i = 0; i < 16; i++)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; i++) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; i++) {
            const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            const uint32_t ch = (e & f) ^ (~e & g);
            const uint32_t t1 = hh + S1 + ch + k[i] + w[i];
            const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
            const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
            const uint32_t t2 = S0 + mj;
            hh = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
    }

    void update(const uint8_t* p, size_t n) {
        total += n;
        if (fill) {
            const size_t take = std::min(n, (size_t)64 - fill);
            std::memcpy(buf + fill, p, take);
            fill += take, p += take, n -= take;
            if (fill == 64) {
                block(buf);
                fill = 0;
            }
        }
        for (; n >= 64; p += 64, n -= 64) block(p);
        if (n) {
            std::memcpy(buf, p, n);
            fill = n;
        }
    }

    std::string hex() {
        const uint64_t bits = total * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; i++) len[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(len, 8);
        static const char* hx = "0123456789abcdef";
        std::string s(64, '0');
        for (int i = 0; i < 8; i++)
            for (int j = 0; j < 4; j++) {
                const uint8_t v = (uint8_t)(h[i] >> (24 - 8 * j));
                s[8 * i + 2 * j] = hx[v >> 4];
                s[8 * i + 2 * j + 1] = hx[v & 15];
            }
        return s;
    }
};

// ---------------------------------------------------------------------------------------------
// A small JSON reader (RFC 8259 values) for the serde_json sections
// ---------------------------------------------------------------------------------------------
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    bool is_uint = false;  // an integer literal that fits u64 exactly
    uint64_t u = 0;
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const char* key) const {
        if (kind != Obj) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JsonParser {
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
    static void utf8(std::string& o, uint32_t c) {
        if (c < 0x80) {
            o += (char)c;
        } else if (c < 0x800) {
            o += (char)(0xC0 | (c >> 6));
            o += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            o += (char)(0xE0 | (c >> 12));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        } else {
            o += (char)(0xF0 | (c >> 18));
            o += (char)(0x80 | ((c >> 12) & 0x3F));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& v) {
        if (end - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    // One UTF-8 sequence whose lead byte c (>= 0x80) was just read, validated as Rust's
    // str::from_utf8 does (RFC 3629: no overlong forms, no surrogates, nothing above U+10FFFF).
    bool utf8_seq(unsigned char c, std::string& o) {
        int n;
        unsigned char lo = 0x80, hi = 0xBF;  // range of the first continuation byte
        if (c >= 0xC2 && c <= 0xDF) n = 1;
        else if (c == 0xE0) n = 2, lo = 0xA0;
        else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) n = 2;
        else if (c == 0xED) n = 2, hi = 0x9F;
        else if (c == 0xF0) n = 3, lo = 0x90;
        else if (c >= 0xF1 && c <= 0xF3) n = 3;
        else if (c == 0xF4) n = 3, hi = 0x8F;
        else return fail("invalid UTF-8 in a string");
        if (end - p < n) return fail("invalid UTF-8 in a string");
        o += (char)c;
        for (int i = 0; i < n; i++) {
            const unsigned char d = (unsigned char)p[i];
            if (d < (i ? 0x80 : lo) || d > (i ? 0xBF : hi)) return fail("invalid UTF-8 in a string");
            o += (char)d;
        }
        p += n;
        return true;
    }
    bool string(std::string& o) {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (p < end && *p != '"') {
            const unsigned char c = (unsigned char)*p++;
            if (c < 0x20) return fail("control character in a string");
            if (c >= 0x80) {
                if (!utf8_seq(c, o)) return false;
                continue;
            }
            if (c != '\\') {
                o += (char)c;
                continue;
            }
            if (p >= end) return fail("truncated escape");
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
                    uint32_t c1;
                    if (!hex4(c1)) return false;
                    if (c1 >= 0xDC00 && c1 < 0xE000) return fail("lone trailing surrogate in a \\u escape");
                    if (c1 >= 0xD800 && c1 < 0xDC00) {  // a high surrogate needs a \\u low surrogate next
                        if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return fail("lone leading surrogate in a \\u escape");
                        p += 2;
                        uint32_t c2;
                        if (!hex4(c2)) return false;
                        if (c2 < 0xDC00 || c2 >= 0xE000) return fail("bad surrogate pair");
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    }
                    utf8(o, c1);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool number(Json& v) {
        const char* s = p;
        if (p < end && *p == '-') p++;
        if (p >= end || *p < '0' || *p > '9') return fail("bad number");
        bool integer = true;
        if (*p == '0' && p + 1 < end && p[1] >= '0' && p[1] <= '9') return fail("bad number (leading zero)");
        while (p < end && *p >= '0' && *p <= '9') p++;
        if (p < end && *p == '.') {
            integer = false;
            p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            integer = false;
            p++;
            if (p < end && (*p == '+' || *p == '-')) p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        const std::string lit(s, p);
        v.kind = Json::Num;
        v.num = strtod(lit.c_str(), nullptr);
        if (integer && lit == "-0") {  // serde_json reads -0 as the integer 0
            v.is_uint = true;
            v.u = 0;
        } else if (integer && lit[0] != '-' && lit.size() <= 20) {
            uint64_t u = 0;
            bool ok = true;
            for (char c : lit) {
                const uint64_t d = (uint64_t)(c - '0');
                if (u > (UINT64_MAX - d) / 10) {
                    ok = false;
                    break;
                }
                u = u * 10 + d;
            }
            v.is_uint = ok;
            v.u = u;
        }
        return true;
    }
    bool value(Json& v) {
        ws();
        if (p >= end) return fail("unexpected end of JSON");
        bool ok = true;
        if ((*p == '{' || *p == '[') && ++depth > 128) return fail("recursion limit exceeded");  // serde_json's
        if (*p == '{') {
            p++;
            v.kind = Json::Obj;
            ws();
            if (p < end && *p == '}') {
                p++;
            } else {
                for (;;) {
                    ws();
                    std::pair<std::string, Json> kv;
                    if (!string(kv.first)) return false;
                    ws();
                    if (p >= end || *p != ':') return fail("expected ':'");
                    p++;
                    if (!value(kv.second)) return false;
                    v.obj.push_back(std::move(kv));
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
            }
        } else if (*p == '[') {
            p++;
            v.kind = Json::Arr;
            ws();
            if (p < end && *p == ']') {
                p++;
            } else {
                for (;;) {
                    Json e;
                    if (!value(e)) return false;
                    v.arr.push_back(std::move(e));
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
            }
        } else if (*p == '"') {
            v.kind = Json::Str;
            ok = string(v.s);
        } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
            v.kind = Json::Bool, v.b = true, p += 4;
        } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
            v.kind = Json::Bool, v.b = false, p += 5;
        } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
            v.kind = Json::Null, p += 4;
        } else {
            ok = number(v);
        }
        if (v.kind == Json::Obj || v.kind == Json::Arr) depth--;
        return ok;
    }
    bool parse(const uint8_t* b, size_t n, Json& out) {
        p = reinterpret_cast<const char*>(b);
        end = p + n;
        if (!value(out)) return false;
        ws();
        if (p != end) return fail("trailing characters after JSON value");
        return true;
    }
};

// ---------------------------------------------------------------------------------------------
// the container
// ---------------------------------------------------------------------------------------------
struct Meta {
    std::string name, sha256;
    int dtype = -1;
    uint32_t group_size = 0;
    std::vector<uint64_t> dims;
    uint64_t data_offset = 0, data_len = 0, scale_offset = 0, scale_len = 0, outlier_offset = 0, outlier_len = 0;
};

int dtype_code(const std::string& s) {
    if (s == "F32") return POX_F32;
    if (s == "F16") return POX_F16;
    if (s == "BF16") return POX_BF16;
    if (s == "I8") return POX_I8;
    if (s == "I4") return POX_I4;
    return -1;  // F8E4M3 / F8E5M2: listed, not served by this backend
}

bool u64_of(const Json* j, uint64_t& v) {
    if (!j || j->kind != Json::Num || !j->is_uint) return false;
    v = j->u;
    return true;
}

// The typed structs the reference deserializes each JSON section into (serde derive, unknown
// fields ignored): PoxMetadata / PoxQuantPlanRecord / PoxManifest / PoxSignatureBlock
// (pox.rs:119-158), ModelConfig (crates/paraoxidizer-core/src/arch.rs:94-112) and TensorMeta
// (crates/paraoxidizer-core/src/tensor.rs:114-128). A section that would not deserialize is a
// format error here as it is an Err there: a missing or repeated field, a wrong JSON type, an
// integer field given a fraction, exponent, sign or out-of-range value, an unknown enum variant.
// (serde would also take a struct written as a JSON array of its fields in order; such a file is
// rejected here.)
enum class FT { Str, OptStr, U64, U32, F64, Bool, MapStr, Arch, DType, Group, Shape, Config };
struct Field {
    const char* key;
    FT type;
    bool required;
};
const Field kConfig[] = {{"architecture", FT::Arch, true},         {"hidden_size", FT::U64, true},
                         {"intermediate_size", FT::U64, true},     {"num_hidden_layers", FT::U64, true},
                         {"num_attention_heads", FT::U64, true},   {"num_key_value_heads", FT::U64, true},
                         {"vocab_size", FT::U64, true},            {"max_position_embeddings", FT::U64, true},
                         {"rms_norm_eps", FT::F64, true},          {"rope_theta", FT::F64, true},
                         {"tie_word_embeddings", FT::Bool, true},  {"eos_token_id", FT::U32, false},
                         {"bos_token_id", FT::U32, false}};
const Field kMetadata[] = {{"model_config", FT::Config, true}, {"total_parameters", FT::U64, true},
                           {"quantized_by", FT::Str, true},    {"timestamp_utc", FT::U64, true},
                           {"original_format", FT::Str, true}, {"base_model_name", FT::Str, true}};
const Field kTensorMeta[] = {{"name", FT::Str, true},         {"shape", FT::Shape, true},
                             {"dtype", FT::DType, true},      {"group_size", FT::Group, true},
                             {"data_offset", FT::U64, true},  {"data_len", FT::U64, true},
                             {"scale_offset", FT::U64, true}, {"scale_len", FT::U64, true},
                             {"outlier_offset", FT::U64, true}, {"outlier_len", FT::U64, true},
                             {"sha256", FT::Str, true}};
const Field kQuantPlan[] = {{"default_precision", FT::Str, true},
                            {"group_size", FT::U64, true},
                            {"outlier_strategy", FT::Str, true},
                            {"layer_assignments", FT::MapStr, true}};
const Field kManifest[] = {{"run_id", FT::Str, true},          {"source_model_sha256", FT::Str, true},
                           {"calibration_sha256", FT::OptStr, false}, {"compiler_version", FT::Str, true},
                           {"target_arch", FT::Str, true},     {"tensor_hashes", FT::MapStr, true},
                           {"artifact_sha256", FT::Str, true}};
const Field kSignature[] = {{"public_key_hex", FT::Str, true}, {"signature_hex", FT::Str, true}};

bool one_of(const std::string& s, std::initializer_list<const char*> names) {
    for (const char* n : names)
        if (s == n) return true;
    return false;
}

template <size_t N>
bool check_struct(const Json& v, const Field (&fields)[N], std::string& err);

bool check_field(const Json& j, FT t, std::string& err) {
    switch (t) {
        case FT::Str: return j.kind == Json::Str;
        case FT::OptStr: return j.kind == Json::Str || j.kind == Json::Null;
        case FT::U64: return j.kind == Json::Num && j.is_uint;
        case FT::U32: return j.kind == Json::Num && j.is_uint && j.u <= 0xFFFFFFFFull;
        case FT::F64: return j.kind == Json::Num && std::isfinite(j.num);
        case FT::Bool: return j.kind == Json::Bool;
        case FT::MapStr:
            if (j.kind != Json::Obj) return false;
            for (const auto& kv : j.obj)
                if (kv.second.kind != Json::Str) return false;
            return true;
        case FT::Arch: return j.kind == Json::Str && one_of(j.s, {"Llama", "Qwen", "Mistral", "Gemma", "Phi", "Custom"});
        case FT::DType:
            return j.kind == Json::Str && one_of(j.s, {"F32", "F16", "BF16", "I8", "I4", "F8E4M3", "F8E5M2"});
        case FT::Group: return j.kind == Json::Str && one_of(j.s, {"None", "G32", "G64", "G128", "G256"});
        case FT::Shape:
            if (j.kind != Json::Arr) return false;
            for (const Json& d : j.arr)
                if (d.kind != Json::Num || !d.is_uint) return false;
            return true;
        case FT::Config: return check_struct(j, kConfig, err);
    }
    return false;
}

template <size_t N>
bool check_struct(const Json& v, const Field (&fields)[N], std::string& err) {
    if (v.kind != Json::Obj) {
        err = "expected a JSON object";
        return false;
    }
    for (const Field& f : fields) {
        const Json* found = nullptr;
        for (const auto& kv : v.obj) {
            if (kv.first != f.key) continue;
            if (found) {
                err = std::string("duplicate field `") + f.key + "`";
                return false;
            }
            found = &kv.second;
        }
        if (!found) {
            if (f.required) {
                err = std::string("missing field `") + f.key + "`";
                return false;
            }
            continue;
        }
        if (!check_field(*found, f.type, err)) {
            if (err.empty()) err = std::string("invalid type or value for `") + f.key + "`";
            return false;
        }
    }
    return true;
}

}  // namespace

struct pox_file {
    const uint8_t* bytes = nullptr;
    size_t len = 0;
    void* map = nullptr;          // mmap'd file (nullptr for from_bytes)
    std::vector<uint8_t> owned;   // from_bytes copies the bytes, as the reference copies them to a temp file
    uint64_t header[12] = {};     // offsets / lengths of the six sections, header order
    uint32_t flags = 0;
    std::vector<Meta> tensors;
    std::map<std::string, size_t> tensor_map;
    Json metadata, quant_plan, manifest;
};

namespace {

uint64_t rd64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; i--) v = v << 8 | p[i];
    return v;
}
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

// Bounds of a section (off, len) inside the file; "out of bounds" is PoxError::Security in the
// reference (pox.rs:188-226).
bool section(const pox_file* f, uint64_t off, uint64_t n, const char* what) {
    if (off > f->len || n > f->len - off) {
        set_error(POX_ERR_FORMAT, "%s out of bounds", what);
        return false;
    }
    return true;
}

bool parse_json(const pox_file* f, uint64_t off, uint64_t n, const char* what, Json& out) {
    if (!section(f, off, n, what)) return false;
    JsonParser jp;
    if (!jp.parse(f->bytes + off, n, out)) {
        set_error(POX_ERR_FORMAT, "%s: invalid JSON (%s)", what, jp.err.c_str());
        return false;
    }
    return true;
}

// PoxFile::from_mmap (pox.rs:248-310): header, then metadata, tensor index, quant plan, manifest and
// signature, each bounds-checked and parsed.
int parse_container(pox_file* f) {
    if (f->len < 128) return set_error(POX_ERR_FORMAT, "File size smaller than header");
    const uint8_t* b = f->bytes;
    if (memcmp(b, "POX\x01", 4) != 0)
        return set_error(POX_ERR_FORMAT, "invalid magic %02x %02x %02x %02x (expected POX\\x01)", b[0], b[1], b[2], b[3]);
    const uint32_t version = rd32(b + 4);
    if (version != 1) return set_error(POX_ERR_FORMAT, "unsupported .pox format version %u", version);
    f->flags = rd32(b + 8);
    for (int i = 0; i < 12; i++) f->header[i] = rd64(b + 16 + 8 * i);
    // header order: metadata, tensor index, quant plan, data, manifest, signature (offset, len each)
    std::string why;
    if (!parse_json(f, f->header[0], f->header[1], "Metadata", f->metadata)) return POX_ERR_FORMAT;
    if (!check_struct(f->metadata, kMetadata, why)) return set_error(POX_ERR_FORMAT, "Metadata: %s", why.c_str());
    Json index;
    if (!parse_json(f, f->header[2], f->header[3], "Tensor index", index)) return POX_ERR_FORMAT;
    if (index.kind != Json::Arr) return set_error(POX_ERR_FORMAT, "tensor index is not a JSON array");
    for (const Json& t : index.arr)
        if (!check_struct(t, kTensorMeta, why)) return set_error(POX_ERR_FORMAT, "Tensor index: %s", why.c_str());
    if (!parse_json(f, f->header[4], f->header[5], "Quant plan", f->quant_plan)) return POX_ERR_FORMAT;
    if (!check_struct(f->quant_plan, kQuantPlan, why)) return set_error(POX_ERR_FORMAT, "Quant plan: %s", why.c_str());
    if (!parse_json(f, f->header[8], f->header[9], "Manifest", f->manifest)) return POX_ERR_FORMAT;
    if (!check_struct(f->manifest, kManifest, why)) return set_error(POX_ERR_FORMAT, "Manifest: %s", why.c_str());
    if (f->header[11] > 0) {
        Json sig;
        if (!parse_json(f, f->header[10], f->header[11], "Signature", sig)) return POX_ERR_FORMAT;
        if (!check_struct(sig, kSignature, why)) return set_error(POX_ERR_FORMAT, "Signature: %s", why.c_str());
    }
    if (!f->metadata.get("model_config") || f->metadata.get("model_config")->kind != Json::Obj)
        return set_error(POX_ERR_FORMAT, "metadata has no model_config");
    if (index.kind != Json::Arr) return set_error(POX_ERR_FORMAT, "tensor index is not a JSON array");
    for (const Json& t : index.arr) {
        Meta m;
        const Json* name = t.get("name");
        const Json* shape = t.get("shape");
        const Json* dtype = t.get("dtype");
        const Json* gs = t.get("group_size");
        const Json* sha = t.get("sha256");
        if (!name || name->kind != Json::Str || !shape || shape->kind != Json::Arr || !dtype ||
            dtype->kind != Json::Str || !gs || gs->kind != Json::Str || !sha || sha->kind != Json::Str)
            return set_error(POX_ERR_FORMAT, "tensor index entry with a missing or mistyped field");
        m.name = name->s;
        m.sha256 = sha->s;
        for (const Json& d : shape->arr) {
            uint64_t v;
            if (!u64_of(&d, v)) return set_error(POX_ERR_FORMAT, "tensor %s: bad shape", m.name.c_str());
            m.dims.push_back(v);
        }
        static const char* dts[] = {"F32", "F16", "BF16", "I8", "I4", "F8E4M3", "F8E5M2"};
        if (std::find_if(std::begin(dts), std::end(dts), [&](const char* d) { return dtype->s == d; }) == std::end(dts))
            return set_error(POX_ERR_FORMAT, "tensor %s: unknown dtype %s", m.name.c_str(), dtype->s.c_str());
        m.dtype = dtype_code(dtype->s);
        if (gs->s == "None") m.group_size = 0;
        else if (gs->s == "G32") m.group_size = 32;
        else if (gs->s == "G64") m.group_size = 64;
        else if (gs->s == "G128") m.group_size = 128;
        else if (gs->s == "G256") m.group_size = 256;
        else return set_error(POX_ERR_FORMAT, "tensor %s: unknown group size %s", m.name.c_str(), gs->s.c_str());
        if (!u64_of(t.get("data_offset"), m.data_offset) || !u64_of(t.get("data_len"), m.data_len) ||
            !u64_of(t.get("scale_offset"), m.scale_offset) || !u64_of(t.get("scale_len"), m.scale_len) ||
            !u64_of(t.get("outlier_offset"), m.outlier_offset) || !u64_of(t.get("outlier_len"), m.outlier_len))
            return set_error(POX_ERR_FORMAT, "tensor %s: bad offsets", m.name.c_str());
        f->tensor_map[m.name] = f->tensors.size();  // a repeated name maps to its last entry, as a HashMap insert
        f->tensors.push_back(std::move(m));
    }
    return POX_OK;
}

// get_tensor_data / get_scale_data / get_outlier_data (pox.rs:311-353): the slice, or NULL when the
// reference returns None (unknown name, an empty scale / outlier section, or a range past the end).
const Meta* find(const pox_file* f, const char* name) {
    if (!f || !name) return nullptr;
    auto it = f->tensor_map.find(name);
    return it == f->tensor_map.end() ? nullptr : &f->tensors[it->second];
}
bool slice(const pox_file* f, uint64_t off, uint64_t n, bool none_if_empty, const uint8_t** p, size_t* len) {
    *p = nullptr;
    *len = 0;
    if (none_if_empty && n == 0) return false;
    if (off > f->len || n > f->len - off) return false;
    *p = f->bytes + off;
    *len = (size_t)n;
    return true;
}
bool data_of(const pox_file* f, const Meta& m, const uint8_t** p, size_t* n) {
    return slice(f, m.data_offset, m.data_len, false, p, n);
}
bool scales_of(const pox_file* f, const Meta& m, const uint8_t** p, size_t* n) {
    return slice(f, m.scale_offset, m.scale_len, true, p, n);
}
bool outliers_of(const pox_file* f, const Meta& m, const uint8_t** p, size_t* n) {
    return slice(f, m.outlier_offset, m.outlier_len, true, p, n);
}

std::string tensor_hash(const pox_file* f, const Meta& m) {
    Sha256 h;
    const uint8_t* p;
    size_t n;
    if (data_of(f, m, &p, &n)) h.update(p, n);
    if (m.scale_len > 0 && scales_of(f, m, &p, &n)) h.update(p, n);
    if (m.outlier_len > 0 && outliers_of(f, m, &p, &n)) h.update(p, n);
    return h.hex();
}

// ---------------------------------------------------------------------------------------------
// tensor-parallel shards of INT4 .pox payloads (the split of the decode model: rows of q, k, v, gate,
// up and lm_head; 128-aligned columns of o and down), outlier tables filtered and re-indexed
// ---------------------------------------------------------------------------------------------
struct Shard {
    std::vector<uint8_t> data, scales, outliers;
    size_t rows = 0, cols = 0;
};

int read_outliers(const uint8_t* b, size_t n, std::vector<uint32_t>& idx, std::vector<uint16_t>& val) {
    idx.clear();
    val.clear();
    if (!b || n < 4) return POX_OK;  // SparseOutlierTable::from_bytes of < 4 bytes: empty (outlier.rs:113-115)
    const uint64_t cnt = rd32(b);
    if (4 + 6 * cnt > n) return set_error(POX_ERR_LAYOUT, "outlier table truncated");
    idx.resize(cnt);
    val.resize(cnt);
    for (uint64_t e = 0; e < cnt; e++) {
        idx[e] = rd32(b + 4 + 4 * e);
        val[e] = (uint16_t)(b[4 + 4 * cnt + 2 * e] | b[4 + 4 * cnt + 2 * e + 1] << 8);
    }
    return POX_OK;
}

void write_outliers(const std::vector<uint32_t>& idx, const std::vector<uint16_t>& val, std::vector<uint8_t>& out) {
    out.clear();
    if (idx.empty()) return;
    const uint32_t cnt = (uint32_t)idx.size();
    out.resize(4 + 6 * (size_t)cnt);
    std::memcpy(out.data(), &cnt, 4);
    std::memcpy(out.data() + 4, idx.data(), 4 * (size_t)cnt);
    std::memcpy(out.data() + 4 + 4 * (size_t)cnt, val.data(), 2 * (size_t)cnt);
}

// split 0: rows [r0, r1); split 1: columns [c0, c1) (multiples of the group size). Index order is kept,
// so the "last entry wins" rule of the replace step (kernels.rs:211-219) holds in every shard.
int shard_i4(const pox_file* f, const Meta& m, int split, uint32_t rank, uint32_t tp, Shard& s) {
    if (m.dtype != POX_I4 || m.dims.size() != 2)
        return set_error(POX_ERR_UNSUPPORTED, "tensor %s: shards are for 2-D INT4 tensors", m.name.c_str());
    const size_t R = m.dims[0], K = m.dims[1], gs = m.group_size;
    if (gs == 0 || K % gs || K % 2) return set_error(POX_ERR_LAYOUT, "tensor %s: groups must line up with rows", m.name.c_str());
    if (tp == 0 || rank >= tp) return set_error(POX_ERR_INVALID, "rank %u of %u", rank, tp);
    const uint8_t *pd, *ps, *po;
    size_t nd, ns, no;
    data_of(f, m, &pd, &nd);
    scales_of(f, m, &ps, &ns);
    outliers_of(f, m, &po, &no);
    const size_t rb = K / 2, sb = K / gs * 4;
    if (!pd || !ps || nd < R * rb || ns < R * sb)
        return set_error(POX_ERR_LAYOUT, "tensor %s: Buffer layout incompatible with 2D GEMV", m.name.c_str());
    std::vector<uint32_t> idx, nidx;
    std::vector<uint16_t> val, nval;
    int rc = read_outliers(po, no, idx, val);
    if (rc) return rc;
    if (split == 0) {
        if (R % tp) return set_error(POX_ERR_UNSUPPORTED, "tensor %s: %zu rows over %u ranks", m.name.c_str(), R, tp);
        const size_t r0 = R / tp * rank, r1 = R / tp * (rank + 1);
        s.rows = r1 - r0;
        s.cols = K;
        s.data.assign(pd + r0 * rb, pd + r1 * rb);
        s.scales.assign(ps + r0 * sb, ps + r1 * sb);
        for (size_t e = 0; e < idx.size(); e++)
            if (idx[e] >= r0 * K && idx[e] < r1 * K) {
                nidx.push_back((uint32_t)(idx[e] - r0 * K));
                nval.push_back(val[e]);
            }
    } else {
        if (K % (gs * tp))
            return set_error(POX_ERR_UNSUPPORTED, "tensor %s: %zu columns over %u ranks in whole groups", m.name.c_str(), K, tp);
        const size_t c0 = K / tp * rank, c1 = K / tp * (rank + 1), w = c1 - c0;
        s.rows = R;
        s.cols = w;
        s.data.resize(R * (w / 2));
        s.scales.resize(R * (w / gs * 4));
        for (size_t r = 0; r < R; r++) {
            std::memcpy(s.data.data() + r * (w / 2), pd + r * rb + c0 / 2, w / 2);
            std::memcpy(s.scales.data() + r * (w / gs * 4), ps + r * sb + c0 / gs * 4, w / gs * 4);
        }
        for (size_t e = 0; e < idx.size(); e++) {
            const size_t r = idx[e] / K, c = idx[e] % K;
            if (r < R && c >= c0 && c < c1) {
                nidx.push_back((uint32_t)(r * w + (c - c0)));
                nval.push_back(val[e]);
            }
        }
    }
    write_outliers(nidx, nval, s.outliers);
    return POX_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------
extern "C" int pox_file_open(const char* path, pox_file** out) {
    if (!path || !out) return set_error(POX_ERR_INVALID, "NULL argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(POX_ERR_INVALID, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return set_error(POX_ERR_INVALID, "cannot stat %s", path);
    }
    auto f = std::make_unique<pox_file>();
    f->len = (size_t)st.st_size;
    if (f->len > 0) {
        void* p = mmap(nullptr, f->len, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            close(fd);
            return set_error(POX_ERR_INVALID, "cannot mmap %s", path);
        }
        f->map = p;
        f->bytes = static_cast<const uint8_t*>(p);
    }
    close(fd);
    const int rc = parse_container(f.get());
    if (rc) {
        if (f->map) munmap(f->map, f->len);
        return rc;
    }
    *out = f.release();
    return POX_OK;
}

extern "C" int pox_file_from_bytes(const uint8_t* bytes, size_t len, pox_file** out) {
    if (!out || (!bytes && len)) return set_error(POX_ERR_INVALID, "NULL argument");
    *out = nullptr;
    auto f = std::make_unique<pox_file>();
    f->owned.assign(bytes, bytes + len);
    f->bytes = f->owned.data();
    f->len = len;
    const int rc = parse_container(f.get());
    if (rc) return rc;
    *out = f.release();
    return POX_OK;
}

extern "C" void pox_file_close(pox_file* f) {
    if (!f) return;
    if (f->map) munmap(f->map, f->len);
    delete f;
}

extern "C" int pox_file_tensor_count(const pox_file* f, size_t* n) {
    if (!f || !n) return set_error(POX_ERR_INVALID, "NULL argument");
    *n = f->tensors.size();
    return POX_OK;
}

extern "C" int pox_file_tensor_meta(const pox_file* f, size_t index, pox_tensor_meta* out) {
    if (!f || !out) return set_error(POX_ERR_INVALID, "NULL argument");
    if (index >= f->tensors.size()) return set_error(POX_ERR_INVALID, "tensor index %zu out of range", index);
    const Meta& m = f->tensors[index];
    *out = pox_tensor_meta{};
    out->name = m.name.c_str();
    out->sha256 = m.sha256.c_str();
    out->dtype = m.dtype;
    out->group_size = m.group_size;
    out->rank = (uint32_t)std::min<size_t>(m.dims.size(), 8);
    for (uint32_t i = 0; i < out->rank; i++) out->dims[i] = m.dims[i];
    out->data_offset = m.data_offset;
    out->data_len = m.data_len;
    out->scale_offset = m.scale_offset;
    out->scale_len = m.scale_len;
    out->outlier_offset = m.outlier_offset;
    out->outlier_len = m.outlier_len;
    return POX_OK;
}

extern "C" int pox_file_find(const pox_file* f, const char* name, size_t* index) {
    if (!f || !name || !index) return set_error(POX_ERR_INVALID, "NULL argument");
    auto it = f->tensor_map.find(name);
    if (it == f->tensor_map.end()) return set_error(POX_ERR_INVALID, "no tensor named %s", name);
    *index = it->second;
    return POX_OK;
}

extern "C" int pox_file_tensor_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len) {
    if (!ptr || !len) return set_error(POX_ERR_INVALID, "NULL argument");
    const Meta* m = find(f, name);
    *ptr = nullptr;
    *len = 0;
    if (m) data_of(f, *m, ptr, len);
    return POX_OK;
}

extern "C" int pox_file_scale_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len) {
    if (!ptr || !len) return set_error(POX_ERR_INVALID, "NULL argument");
    const Meta* m = find(f, name);
    *ptr = nullptr;
    *len = 0;
    if (m) scales_of(f, *m, ptr, len);
    return POX_OK;
}

extern "C" int pox_file_outlier_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len) {
    if (!ptr || !len) return set_error(POX_ERR_INVALID, "NULL argument");
    const Meta* m = find(f, name);
    *ptr = nullptr;
    *len = 0;
    if (m) outliers_of(f, *m, ptr, len);
    return POX_OK;
}

extern "C" int pox_file_model_config(const pox_file* f, pox_llama_config* cfg, int* tie_word_embeddings) {
    if (!f || !cfg) return set_error(POX_ERR_INVALID, "NULL argument");
    const Json* mc = f->metadata.get("model_config");
    uint64_t h, i, l, nh, nkv, v;
    if (!u64_of(mc->get("hidden_size"), h) || !u64_of(mc->get("intermediate_size"), i) ||
        !u64_of(mc->get("num_hidden_layers"), l) || !u64_of(mc->get("num_attention_heads"), nh) ||
        !u64_of(mc->get("num_key_value_heads"), nkv) || !u64_of(mc->get("vocab_size"), v))
        return set_error(POX_ERR_FORMAT, "model_config: missing or non-integer size field");
    const Json* eps = mc->get("rms_norm_eps");
    const Json* theta = mc->get("rope_theta");
    if (!eps || eps->kind != Json::Num || !theta || theta->kind != Json::Num)
        return set_error(POX_ERR_FORMAT, "model_config: rms_norm_eps / rope_theta missing");
    if (h > UINT32_MAX || i > UINT32_MAX || l > UINT32_MAX || nh > UINT32_MAX || nkv > UINT32_MAX || v > UINT32_MAX)
        return set_error(POX_ERR_UNSUPPORTED, "model_config: a size beyond 2^32");
    cfg->hidden = (uint32_t)h;
    cfg->intermediate = (uint32_t)i;
    cfg->layers = (uint32_t)l;
    cfg->heads = (uint32_t)nh;
    cfg->kv_heads = (uint32_t)nkv;
    cfg->vocab = (uint32_t)v;
    cfg->rms_eps = (float)eps->num;  // the engine reads them as f32 (engine.rs:535, 353-408)
    cfg->rope_theta = (float)theta->num;
    if (tie_word_embeddings) {
        const Json* t = mc->get("tie_word_embeddings");
        *tie_word_embeddings = t && t->kind == Json::Bool && t->b;
    }
    return POX_OK;
}

extern "C" int pox_file_verify_integrity(const pox_file* f, int threads) {
    if (!f) return set_error(POX_ERR_INVALID, "file is NULL");
    const size_t n = f->tensors.size();
    for (const Meta& m : f->tensors) {
        const uint8_t* p;
        size_t len;
        if (!data_of(f, m, &p, &len)) return set_error(POX_ERR_FORMAT, "Missing data for tensor %s", m.name.c_str());
    }
    std::vector<std::string> got(n);
    unsigned nt = threads > 0 ? (unsigned)threads : std::max(1u, std::thread::hardware_concurrency());
    nt = (unsigned)std::min<size_t>(nt, std::max<size_t>(n, 1));
    std::atomic<size_t> next{0};
    auto work = [&] {
        for (size_t i; (i = next++) < n;) got[i] = tensor_hash(f, f->tensors[i]);
    };
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < nt; t++) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    for (size_t i = 0; i < n; i++)  // the first mismatch in index order, as the reference's loop reports it
        if (got[i] != f->tensors[i].sha256)
            return set_error(POX_ERR_INTEGRITY, "integrity hash mismatch for tensor %s: expected %s, calculated %s",
                             f->tensors[i].name.c_str(), f->tensors[i].sha256.c_str(), got[i].c_str());
    return POX_OK;
}

extern "C" int pox_file_tensor_shard(const pox_file* f, const char* name, int split, uint32_t tp_rank, uint32_t tp_size,
                                     uint8_t* data, size_t* data_len, uint8_t* scales, size_t* scale_len,
                                     uint8_t* outliers, size_t* outlier_len) {
    if (!f || !name || !data_len || !scale_len || !outlier_len) return set_error(POX_ERR_INVALID, "NULL argument");
    if (split != 0 && split != 1) return set_error(POX_ERR_INVALID, "split must be 0 (rows) or 1 (columns)");
    const Meta* m = find(f, name);
    if (!m) return set_error(POX_ERR_INVALID, "no tensor named %s", name);
    Shard s;
    const int rc = shard_i4(f, *m, split, tp_rank, tp_size, s);
    if (rc) return rc;
    const bool fits = data && scales && (outliers || s.outliers.empty()) && *data_len >= s.data.size() &&
                      *scale_len >= s.scales.size() && *outlier_len >= s.outliers.size();
    if (fits) {
        std::memcpy(data, s.data.data(), s.data.size());
        std::memcpy(scales, s.scales.data(), s.scales.size());
        if (!s.outliers.empty()) std::memcpy(outliers, s.outliers.data(), s.outliers.size());
    }
    *data_len = s.data.size();
    *scale_len = s.scales.size();
    *outlier_len = s.outliers.size();
    return fits ? POX_OK : set_error(POX_ERR_LAYOUT, "shard buffers too small (sizes returned)");
}

// The decode model of a .pox file (engine.rs tensor names, :424-713): embedding, final norm and lm_head
// as F16, per layer the seven INT4 projections (optional outlier tables) and two F16 norms; rank tp_rank
// of tp_size takes its shards (pox_cuda_model_create_tp). Payloads are read from the mmap once and
// uploaded; the file may be closed afterwards.
extern "C" int pox_cuda_model_load(pox_cuda_ctx* ctx, const pox_file* f, uint32_t max_batch, uint32_t kv_blocks,
                                   uint32_t max_blocks_per_seq, uint32_t tp_rank, uint32_t tp_size, pox_model** out) {
    if (!ctx || !f || !out) return set_error(POX_ERR_INVALID, "NULL argument");
    *out = nullptr;
    pox_llama_config cfg;
    int tie = 0;
    int rc = pox_file_model_config(f, &cfg, &tie);
    if (rc) return rc;
    auto f16 = [&](const std::string& name, size_t n, const uint8_t** p) -> int {
        const Meta* m = find(f, name.c_str());
        if (!m) return set_error(POX_ERR_FORMAT, "tensor %s missing", name.c_str());
        if (m->dtype != POX_F16)
            return set_error(POX_ERR_UNSUPPORTED, "tensor %s: the CUDA decode path takes it as F16", name.c_str());
        size_t len;
        if (!data_of(f, *m, p, &len) || len < n * 2)
            return set_error(POX_ERR_LAYOUT, "tensor %s: %zu bytes, need %zu", name.c_str(), len, n * 2);
        return POX_OK;
    };
    const size_t H = cfg.hidden, V = cfg.vocab;
    const uint8_t *embed, *final_norm, *head;
    if ((rc = f16("model.embed_tokens.weight", V * H, &embed))) return rc;
    if ((rc = f16("model.norm.weight", H, &final_norm))) return rc;
    const bool has_head = find(f, "lm_head.weight") != nullptr;
    if (!has_head && !tie) return set_error(POX_ERR_FORMAT, "tensor lm_head.weight missing");
    if ((rc = f16(has_head ? "lm_head.weight" : "model.embed_tokens.weight", V * H, &head))) return rc;
    pox_model* m = nullptr;
    if ((rc = pox_cuda_model_create_tp(ctx, &cfg, max_batch, kv_blocks, max_blocks_per_seq, tp_rank, tp_size, &m)))
        return rc;
    auto fail = [&](int code) {
        pox_cuda_model_destroy(m);
        return code;
    };
    static const char* proj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                  "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"};
    static const int split[7] = {0, 0, 0, 1, 0, 0, 1};
    for (uint32_t l = 0; l < cfg.layers; l++) {
        Shard sh[7];
        pox_tensor_desc d[7];
        for (int j = 0; j < 7; j++) {
            const std::string name = "model.layers." + std::to_string(l) + "." + proj[j] + ".weight";
            const Meta* t = find(f, name.c_str());
            if (!t) return fail(set_error(POX_ERR_FORMAT, "tensor %s missing", name.c_str()));
            if (t->dtype != POX_I4)
                return fail(set_error(POX_ERR_UNSUPPORTED, "tensor %s: the CUDA decode path takes INT4 projections",
                                      name.c_str()));
            if ((rc = shard_i4(f, *t, split[j], tp_rank, tp_size, sh[j]))) return fail(rc);
            d[j] = pox_tensor_desc{};
            d[j].dtype = POX_I4;
            d[j].rows = sh[j].rows;
            d[j].cols = sh[j].cols;
            d[j].group_size = t->group_size;
            d[j].data = sh[j].data.data();
            d[j].data_len = sh[j].data.size();
            d[j].scales = sh[j].scales.data();
            d[j].scale_len = sh[j].scales.size();
            d[j].outliers = sh[j].outliers.empty() ? nullptr : sh[j].outliers.data();
            d[j].outlier_len = sh[j].outliers.size();
        }
        const uint8_t *an, *mn;
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        if ((rc = f16(pre + "input_layernorm.weight", H, &an))) return fail(rc);
        if ((rc = f16(pre + "post_attention_layernorm.weight", H, &mn))) return fail(rc);
        if ((rc = pox_cuda_model_set_layer(m, l, d, reinterpret_cast<const uint16_t*>(an),
                                           reinterpret_cast<const uint16_t*>(mn))))
            return fail(rc);
    }
    const size_t Vl = V / tp_size;
    if ((rc = pox_cuda_model_set_embeddings(m, reinterpret_cast<const uint16_t*>(embed),
                                            reinterpret_cast<const uint16_t*>(final_norm),
                                            reinterpret_cast<const uint16_t*>(head + Vl * tp_rank * H * 2))))
        return fail(rc);
    *out = m;
    return POX_OK;
}
