// FORGEMODEL1 checkpoints (src/LLM.Core/Checkpoint/Checkpoint.cs), host side.
//
// File layout (Checkpoint.WriteHeaderAndWeights, Checkpoint.cs:143-166):
//   "FORGEMODEL1" (11 bytes) | int32 LE header length n (0 < n <= 2^20) |
//   n bytes of UTF-8 JSON {VocabSize, ContextLength, DModel, NLayers, NHeads,
//   ModelName, Architecture, Names[], Training{..., HasOptimizerState, ...}} |
//   every parameter in registry order as fp32 LE | when HasOptimizerState, per
//   parameter its Adam m then v tensors | SHA-256 of all preceding bytes.
// Checkpoint.LoadCore (Checkpoint.cs:174-264) rejects: a wrong magic, a file
// too short for its checksum, an implausible header length, a header that
// does not parse, an architecture other than "forge-gpt2-tied-v1", an empty
// model name, a missing Training object, parameter names that differ from the
// registry, a payload of the wrong size, a checksum mismatch, trailing data.
// This file restates those rules; SHA-256 follows FIPS 180-4.
#pragma once
#include <algorithm>
#include <cerrno>
#include <climits>
#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace fb2 {
namespace fm {

// ---- SHA-256 (FIPS 180-4) -------------------------------------------------------
// The round constants are the first 32 fractional bits of the cube roots of the
// first 64 primes, the initial hash the same of the square roots of the first
// 8 primes (FIPS 180-4 4.2.2, 5.3.3); computed here with exact integer roots.
class Sha256 {
public:
    Sha256() {
        const Tables& t = tables();
        std::memcpy(h_, t.h0, sizeof h_);
    }
    void update(const void* data, size_t n) {
        const unsigned char* p = static_cast<const unsigned char*>(data);
        total_ += n;
        if (fill_) {
            size_t take = std::min(n, (size_t)64 - fill_);
            std::memcpy(buf_ + fill_, p, take);
            fill_ += take;
            p += take;
            n -= take;
            if (fill_ == 64) {
                block(buf_);
                fill_ = 0;
            }
        }
        while (n >= 64) {
            block(p);
            p += 64;
            n -= 64;
        }
        if (n) {
            std::memcpy(buf_, p, n);
            fill_ = n;
        }
    }
    void finish(unsigned char out[32]) {
        const uint64_t bits = total_ * 8;
        unsigned char pad[72] = {0x80};
        const size_t padlen = (fill_ < 56) ? 56 - fill_ : 120 - fill_;
        update(pad, padlen);
        unsigned char len[8];
        for (int i = 0; i < 8; i++) len[i] = (unsigned char)(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; i++)
            for (int j = 0; j < 4; j++) out[4 * i + j] = (unsigned char)(h_[i] >> (24 - 8 * j));
    }

private:
    struct Tables {
        uint32_t k[64], h0[8];
    };
    static unsigned __int128 iroot(unsigned __int128 n, int e) {  // floor(n^(1/e)), e in {2, 3}
        unsigned __int128 lo = 0, hi = (unsigned __int128)1 << (e == 2 ? 64 : 43);
        while (lo < hi) {
            unsigned __int128 mid = (lo + hi + 1) >> 1, p = mid * mid;
            if (e == 3) p *= mid;
            if (p <= n) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    }
    static const Tables& tables() {
        static const Tables t = [] {
            Tables r{};
            int primes[64], np = 0;
            for (int c = 2; np < 64; c++) {
                bool prime = true;
                for (int d = 2; d * d <= c; d++)
                    if (c % d == 0) prime = false;
                if (prime) primes[np++] = c;
            }
            for (int i = 0; i < 64; i++)
                r.k[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 96, 3);
            for (int i = 0; i < 8; i++) r.h0[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 64, 2);
            return r;
        }();
        return t;
    }
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
    void block(const unsigned char* p) {
        const Tables& t = tables();
        uint32_t w[64];
        for (int i = 0; i < 16; i++)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; i++) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
        for (int i = 0; i < 64; i++) {
            const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            const uint32_t ch = (e & f) ^ (~e & g);
            const uint32_t t1 = h + S1 + ch + t.k[i] + w[i];
            const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
            const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
            const uint32_t t2 = S0 + mj;
            h = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
    }
    uint32_t h_[8];
    unsigned char buf_[64];
    size_t fill_ = 0;
    uint64_t total_ = 0;
};

// ---- minimal JSON ----------------------------------------------------------------
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    long long inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;
    const Json* get(const std::string& k) const {
        auto it = obj.find(k);
        return kind == Obj && it != obj.end() ? &it->second : nullptr;
    }
};

class JsonParser {
public:
    JsonParser(const char* p, size_t n) : p_(p), e_(p + n) {}
    Json parse() {
        Json v = value(0);
        ws();
        if (p_ != e_) throw std::runtime_error("trailing characters after the JSON value");
        return v;
    }

private:
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
    }
    [[noreturn]] void bad(const char* what) { throw std::runtime_error(std::string("JSON: ") + what); }
    bool lit(const char* s) {
        size_t n = std::strlen(s);
        if ((size_t)(e_ - p_) >= n && std::memcmp(p_, s, n) == 0) {
            p_ += n;
            return true;
        }
        return false;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) out += (char)cp;
        else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (e_ - p_ < 4) bad("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else bad("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        if (p_ >= e_ || *p_ != '"') bad("expected a string");
        p_++;
        std::string out;
        while (true) {
            if (p_ >= e_) bad("unterminated string");
            const char c = *p_++;
            if (c == '"') break;
            if ((unsigned char)c < 0x20) bad("control character in a string");
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p_ >= e_) bad("unterminated escape");
            const char x = *p_++;
            switch (x) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                uint32_t cp = hex4();
                if (cp >= 0xD800 && cp < 0xDC00) {
                    if (!(e_ - p_ >= 2 && p_[0] == '\\' && p_[1] == 'u')) bad("unpaired surrogate");
                    p_ += 2;
                    const uint32_t lo = hex4();
                    if (lo < 0xDC00 || lo >= 0xE000) bad("unpaired surrogate");
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                }
                utf8(out, cp);
                break;
            }
            default: bad("unknown escape");
            }
        }
        return out;
    }
    Json value(int depth) {
        if (depth > 64) bad("nesting too deep");
        ws();
        if (p_ >= e_) bad("unexpected end");
        Json v;
        const char c = *p_;
        if (c == '{') {
            p_++;
            v.kind = Json::Obj;
            ws();
            if (p_ < e_ && *p_ == '}') {
                p_++;
                return v;
            }
            while (true) {
                ws();
                std::string k = string();
                ws();
                if (p_ >= e_ || *p_ != ':') bad("expected ':'");
                p_++;
                v.obj[k] = value(depth + 1);
                ws();
                if (p_ < e_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < e_ && *p_ == '}') {
                    p_++;
                    return v;
                }
                bad("expected ',' or '}'");
            }
        }
        if (c == '[') {
            p_++;
            v.kind = Json::Arr;
            ws();
            if (p_ < e_ && *p_ == ']') {
                p_++;
                return v;
            }
            while (true) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (p_ < e_ && *p_ == ',') {
                    p_++;
                    continue;
                }
                if (p_ < e_ && *p_ == ']') {
                    p_++;
                    return v;
                }
                bad("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::Str;
            v.str = string();
            return v;
        }
        if (lit("true")) {
            v.kind = Json::Bool;
            v.b = true;
            return v;
        }
        if (lit("false")) {
            v.kind = Json::Bool;
            return v;
        }
        if (lit("null")) return v;
        // number
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') p_++;
        bool frac = false;
        while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                           *p_ == '-')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') frac = true;
            p_++;
        }
        if (p_ == s) bad("unexpected character");
        const std::string t(s, p_);
        char* end = nullptr;
        v.kind = Json::Num;
        v.num = std::strtod(t.c_str(), &end);
        if (!end || *end) bad("bad number");
        if (!frac) {
            errno = 0;
            v.inum = std::strtoll(t.c_str(), &end, 10);
            v.is_int = errno == 0 && end && !*end;
        }
        return v;
    }
    const char* p_;
    const char* e_;
};

inline std::string json_escape(const std::string& s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c < 0x20) {
            char b[8];
            std::snprintf(b, sizeof b, "\\u%04x", c);
            o += b;
        } else o += (char)c;
    }
    return o + "\"";
}

constexpr const char kMagic[] = "FORGEMODEL1";
constexpr size_t kMagicLen = 11;
constexpr const char kArchitecture[] = "forge-gpt2-tied-v1";

// The parameter registry names in Parameters.Names order (GptModel.cs:14-18,
// Layers.cs registrations): tok_emb, pos_emb, blocks.i.{...}, ln_f.w, ln_f.b.
inline std::vector<std::string> registry_names(int n_layers) {
    std::vector<std::string> n = {"tok_emb", "pos_emb"};
    static const char* block[12] = {"ln1.w",    "ln1.b",    "attn.qkv.w", "attn.qkv.b", "attn.proj.w", "attn.proj.b",
                                    "ln2.w",    "ln2.b",    "mlp.fc.w",   "mlp.fc.b",   "mlp.proj.w",  "mlp.proj.b"};
    for (int l = 0; l < n_layers; l++)
        for (const char* b : block) n.push_back("blocks." + std::to_string(l) + "." + b);
    n.push_back("ln_f.w");
    n.push_back("ln_f.b");
    return n;
}

struct Header {
    int vocab = 0, ctx = 0, d_model = 0, n_layers = 0, n_heads = 0;
    std::string name;
    bool moments = false;
};

// Thrown for every rule of Checkpoint.LoadCore; maps to FB2_INVALID_DATA.
struct InvalidData : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// A validated checkpoint held in memory: header + the weights' byte offset.
struct File {
    Header hdr;
    std::vector<unsigned char> bytes;
    size_t weights_at = 0;
};

// Parameter count of the registry (GptModel.cs:38-99): embeddings, 12D^2 + 13D
// per block, ln_f.
inline long long param_count(const Header& h) {
    const long long D = h.d_model;
    return (long long)h.vocab * D + (long long)h.ctx * D + (long long)h.n_layers * (12 * D * D + 13 * D) + 2 * D;
}

inline File read_file(const char* path) {
    File f;
    {
        std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path, "rb"), std::fclose);
        if (!fp) throw std::runtime_error(std::string("cannot open '") + path + "'");
        if (std::fseek(fp.get(), 0, SEEK_END) != 0) throw std::runtime_error("cannot seek the checkpoint");
        const long size = std::ftell(fp.get());
        if (size < 0) throw std::runtime_error("cannot size the checkpoint");
        std::rewind(fp.get());
        f.bytes.resize((size_t)size);
        if (size && std::fread(f.bytes.data(), 1, (size_t)size, fp.get()) != (size_t)size)
            throw std::runtime_error("short read of the checkpoint");
    }
    const std::vector<unsigned char>& b = f.bytes;
    if (b.size() < kMagicLen || std::memcmp(b.data(), kMagic, kMagicLen) != 0)
        throw InvalidData(std::string("'") + path + "' is not a current FORGEMODEL1 checkpoint.");
    if (b.size() < kMagicLen + 32) throw InvalidData("Checkpoint is too short to contain its checksum.");
    const size_t content = b.size() - 32;
    if (content < kMagicLen + 4) throw InvalidData("Checkpoint ended inside its JSON header.");
    int32_t jlen;
    std::memcpy(&jlen, b.data() + kMagicLen, 4);
    if (jlen <= 0 || jlen > (1 << 20)) throw InvalidData("Implausible header length " + std::to_string(jlen) + ".");
    const size_t jat = kMagicLen + 4;
    if (jat + (size_t)jlen > content) throw InvalidData("Checkpoint ended inside its JSON header.");
    Json j;
    try {
        j = JsonParser(reinterpret_cast<const char*>(b.data() + jat), (size_t)jlen).parse();
    } catch (const std::runtime_error& e) {
        throw InvalidData(std::string("Checkpoint header failed to parse: ") + e.what());
    }
    if (j.kind != Json::Obj) throw InvalidData("Checkpoint header failed to parse.");
    auto geti = [&](const char* k) -> int {
        const Json* v = j.get(k);
        if (!v || v->kind != Json::Num || !v->is_int || v->inum < INT32_MIN || v->inum > INT32_MAX)
            throw InvalidData(std::string("Checkpoint header field ") + k + " is missing or not an integer.");
        return (int)v->inum;
    };
    Header& h = f.hdr;
    h.vocab = geti("VocabSize");
    h.ctx = geti("ContextLength");
    h.d_model = geti("DModel");
    h.n_layers = geti("NLayers");
    h.n_heads = geti("NHeads");
    const Json* arch = j.get("Architecture");
    if (!arch || arch->kind != Json::Str || arch->str != kArchitecture)
        throw InvalidData("Unsupported checkpoint architecture '" + (arch && arch->kind == Json::Str ? arch->str : "") +
                          "'.");
    const Json* name = j.get("ModelName");
    bool blank = !name || name->kind != Json::Str;
    if (!blank) {
        blank = true;
        for (char c : name->str)
            if (!(c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f')) blank = false;
    }
    if (blank) throw InvalidData("Checkpoint is missing its Forge model name.");
    h.name = name->str;
    const Json* tr = j.get("Training");
    if (!tr || tr->kind != Json::Obj) throw InvalidData("Training checkpoint is missing its training-state header.");
    const Json* hm = tr->get("HasOptimizerState");
    h.moments = hm && hm->kind == Json::Bool && hm->b;
    // ModelConfig validation (ModelConfig.cs:8-26)
    if (h.vocab <= 0 || h.ctx <= 0 || h.d_model <= 0 || h.n_layers <= 0 || h.n_heads <= 0 || h.d_model % h.n_heads)
        throw InvalidData("Checkpoint model configuration is invalid.");
    const Json* names = j.get("Names");
    const std::vector<std::string> want = registry_names(h.n_layers);
    bool same = names && names->kind == Json::Arr && names->arr.size() == want.size();
    for (size_t i = 0; same && i < want.size(); i++)
        same = names->arr[i].kind == Json::Str && names->arr[i].str == want[i];
    if (!same) throw InvalidData("Checkpoint parameter names do not match the model registry.");
    f.weights_at = jat + (size_t)jlen;
    const unsigned long long wbytes = (unsigned long long)param_count(h) * 4ull;
    const unsigned long long expect = wbytes * (h.moments ? 3ull : 1ull);
    if ((unsigned long long)(content - f.weights_at) != expect)
        throw InvalidData("Checkpoint payload is " + std::to_string(content - f.weights_at) + " bytes, expected " +
                          std::to_string(expect) + ".");
    Sha256 sha;
    sha.update(b.data(), content);
    unsigned char digest[32];
    sha.finish(digest);
    if (std::memcmp(digest, b.data() + content, 32) != 0)
        throw InvalidData("Checkpoint SHA-256 checksum does not match; the file is corrupted.");
    return f;
}

// Model checkpoint in the format Checkpoint.SaveTraining writes, with a
// Training header that records no optimizer state (inference weights only).
inline void write_file(const char* path, const Header& h, const float* const* params, int n_params) {
    const std::vector<std::string> names = registry_names(h.n_layers);
    if ((int)names.size() != n_params) throw std::invalid_argument("n_params does not match the registry");
    std::string js = "{\"VocabSize\":" + std::to_string(h.vocab) + ",\"ContextLength\":" + std::to_string(h.ctx) +
                     ",\"DModel\":" + std::to_string(h.d_model) + ",\"NLayers\":" + std::to_string(h.n_layers) +
                     ",\"NHeads\":" + std::to_string(h.n_heads) + ",\"ModelName\":" + json_escape(h.name) +
                     ",\"Architecture\":" + json_escape(kArchitecture) + ",\"Names\":[";
    for (size_t i = 0; i < names.size(); i++) js += (i ? "," : "") + json_escape(names[i]);
    js += "],\"Training\":{\"GlobalStep\":0,\"AdamStep\":0,\"SamplerRandomState\":0,\"SamplerRandomIncrement\":0,"
          "\"SamplerEpoch\":0,\"SamplerCursor\":0,\"SamplerStart\":0,\"SamplerStride\":0,\"SamplerChunkCount\":0,"
          "\"SamplerContextLength\":0,\"HasOptimizerState\":false,\"TotalSteps\":0,\"MaxLr\":0,\"MinLr\":0,"
          "\"WarmupSteps\":0,\"WeightDecay\":0,\"GradClip\":0,\"BatchSize\":0,\"AccumulationSteps\":0,"
          "\"TrainingContextLength\":0,\"DataIdentity\":null,\"TokenizerIdentity\":null}}";
    std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path, "wb"), std::fclose);
    if (!fp) throw std::runtime_error(std::string("cannot create '") + path + "'");
    Sha256 sha;
    auto put = [&](const void* p, size_t n) {
        if (n && std::fwrite(p, 1, n, fp.get()) != n) throw std::runtime_error("short write of the checkpoint");
        sha.update(p, n);
    };
    put(kMagic, kMagicLen);
    const int32_t jlen = (int32_t)js.size();
    put(&jlen, 4);
    put(js.data(), js.size());
    const long long D = h.d_model;
    std::vector<long long> numel = {(long long)h.vocab * D, (long long)h.ctx * D};
    for (int l = 0; l < h.n_layers; l++) {
        const long long b[12] = {D, D, 3 * D * D, 3 * D, D * D, D, D, D, 4 * D * D, 4 * D, 4 * D * D, D};
        numel.insert(numel.end(), b, b + 12);
    }
    numel.push_back(D);
    numel.push_back(D);
    for (int i = 0; i < n_params; i++) put(params[i], (size_t)numel[i] * 4);
    unsigned char digest[32];
    sha.finish(digest);
    if (std::fwrite(digest, 1, 32, fp.get()) != 32) throw std::runtime_error("short write of the checkpoint");
    if (std::fflush(fp.get()) != 0) throw std::runtime_error("cannot flush the checkpoint");
}

}  // namespace fm
}  // namespace fb2
