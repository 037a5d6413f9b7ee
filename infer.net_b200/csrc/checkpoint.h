// MLX checkpoint reading for the MoE block: config.json, model.safetensors.index.json and the
// safetensors shards it names (host code only; no CUDA).
//
// The reference reads the same files in Qwen36Weights (src/DeepInfer.Backends/Models/
// Qwen36Weights.cs:55-100) through SafeTensors (src/DeepInfer.Backends/Models/SafeTensors.cs:13-46):
// a bounded JSON header of typed tensors (BF16, F32, U32) with validated shapes and non-overlapping
// byte ranges, shard file names that cannot leave the directory, and per-matrix quantisation
// overrides that must agree with the expected bits. This file implements those rules in C++ with its
// own small JSON reader (strings, numbers, objects, arrays, literals).
#pragma once

#include <sys/types.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace di {
namespace ckpt {

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// ------------------------------------------------------------------ JSON

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;  // in document order

    const Json *get(const std::string &key) const {
        if (kind != Object) return nullptr;
        for (const auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    const Json &at(const std::string &key, const char *what) const {
        const Json *v = get(key);
        if (!v) throw Error(std::string("Missing ") + what + " '" + key + "'.");
        return *v;
    }
    int64_t as_int(const char *what) const {
        if (kind != Number || num != (double)(int64_t)num) throw Error(std::string("Expected an integer for ") + what + ".");
        return (int64_t)num;
    }
    const std::string &as_str(const char *what) const {
        if (kind != String) throw Error(std::string("Expected a string for ") + what + ".");
        return str;
    }
};

class JsonReader {
public:
    JsonReader(const char *s, size_t n) : p_(s), end_(s + n) {}
    Json document() {
        Json v = value(0);
        ws();
        if (p_ != end_) fail("trailing characters");
        return v;
    }

private:
    const char *p_, *end_;
    [[noreturn]] void fail(const char *why) { throw Error(std::string("Invalid JSON: ") + why + "."); }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char *w) {
        const size_t n = std::strlen(w);
        if ((size_t)(end_ - p_) >= n && std::memcmp(p_, w, n) == 0) {
            p_ += n;
            return true;
        }
        return false;
    }
    Json value(int depth) {
        if (depth > 64) fail("nesting too deep");
        ws();
        if (p_ >= end_) fail("unexpected end");
        Json v;
        const char c = *p_;
        if (c == '{') {
            v.kind = Json::Object;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return v;
            }
            for (;;) {
                ws();
                if (p_ >= end_ || *p_ != '"') fail("expected a key");
                std::string key = string();
                ws();
                if (p_ >= end_ || *p_ != ':') fail("expected ':'");
                ++p_;
                v.obj.emplace_back(std::move(key), value(depth + 1));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::Array;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return v;
            }
            for (;;) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::String;
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
        if (c == '-' || (c >= '0' && c <= '9')) {
            const char *s = p_;
            if (*p_ == '-') ++p_;
            while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                                 *p_ == '-'))
                ++p_;
            std::string t(s, p_);
            char *e = nullptr;
            v.kind = Json::Number;
            v.num = std::strtod(t.c_str(), &e);
            if (!e || *e) fail("bad number");
            return v;
        }
        fail("unexpected character");
    }
    std::string string() {
        ++p_;  // opening quote
        std::string out;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (p_ >= end_) fail("bad escape");
            const char e = *p_++;
            switch (e) {
            case '"': out.push_back('"'); break;
            case '\\': out.push_back('\\'); break;
            case '/': out.push_back('/'); break;
            case 'b': out.push_back('\b'); break;
            case 'f': out.push_back('\f'); break;
            case 'n': out.push_back('\n'); break;
            case 'r': out.push_back('\r'); break;
            case 't': out.push_back('\t'); break;
            case 'u': {
                if (end_ - p_ < 4) fail("bad \\u escape");
                unsigned cp = 0;
                for (int i = 0; i < 4; ++i) {
                    const char h = *p_++;
                    const int d = h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                                       : h >= 'A' && h <= 'F' ? h - 'A' + 10 : -1;
                    if (d < 0) fail("bad \\u escape");
                    cp = cp * 16 + (unsigned)d;
                }
                // UTF-8 of the code unit (names in checkpoints are ASCII; surrogates are kept as-is)
                if (cp < 0x80) out.push_back((char)cp);
                else if (cp < 0x800) {
                    out.push_back((char)(0xC0 | (cp >> 6)));
                    out.push_back((char)(0x80 | (cp & 0x3F)));
                } else {
                    out.push_back((char)(0xE0 | (cp >> 12)));
                    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
                    out.push_back((char)(0x80 | (cp & 0x3F)));
                }
                break;
            }
            default: fail("bad escape");
            }
        }
        if (p_ >= end_) fail("unterminated string");
        ++p_;
        return out;
    }
};

inline std::vector<char> read_file(const std::string &path, size_t limit) {
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) throw Error("Cannot open " + path + ".");
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (n < 0 || (size_t)n > limit) {
        std::fclose(f);
        throw Error("Unexpected size of " + path + ".");
    }
    std::vector<char> buf((size_t)n);
    const size_t got = n ? std::fread(buf.data(), 1, (size_t)n, f) : 0;
    std::fclose(f);
    if (got != (size_t)n) throw Error("Cannot read " + path + ".");
    return buf;
}

inline Json parse_file(const std::string &path) {
    const std::vector<char> b = read_file(path, 64u << 20);
    return JsonReader(b.data(), b.size()).document();
}

// ------------------------------------------------------------------ safetensors

struct Tensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t start = 0, bytes = 0;  // absolute file offset and length
};

// One shard: its header, validated as SafeTensors.cs:18-44 does (header length in [2, 16 MiB] and
// within the file; dtypes BF16, F32, U32; 1 to 8 positive dimensions; byte ranges inside the data
// area, of the size the shape implies, unique names, no overlaps).
class Shard {
public:
    explicit Shard(const std::string &path) : path_(path) {
        FILE *f = std::fopen(path.c_str(), "rb");
        if (!f) throw Error("Cannot open shard " + path + ".");
        std::fseek(f, 0, SEEK_END);
        const long size = std::ftell(f);
        std::fseek(f, 0, SEEK_SET);
        uint8_t lb[8];
        if (size < 8 || std::fread(lb, 1, 8, f) != 8) {
            std::fclose(f);
            throw Error("Invalid safetensors header length.");
        }
        uint64_t hl = 0;
        for (int i = 7; i >= 0; --i) hl = (hl << 8) | lb[i];
        if (hl < 2 || hl > (16u << 20) || hl > (uint64_t)size - 8) {
            std::fclose(f);
            throw Error("Invalid safetensors header length.");
        }
        std::vector<char> hdr((size_t)hl);
        const size_t got = std::fread(hdr.data(), 1, hdr.size(), f);
        std::fclose(f);
        if (got != hdr.size()) throw Error("Invalid safetensors header length.");
        const uint64_t data0 = 8 + hl, data_bytes = (uint64_t)size - data0;
        const Json j = JsonReader(hdr.data(), hdr.size()).document();
        if (j.kind != Json::Object) throw Error("Invalid safetensors header.");
        std::vector<std::pair<uint64_t, uint64_t>> ranges;
        for (const auto &kv : j.obj) {
            if (kv.first == "__metadata__") continue;
            const Json &v = kv.second;
            Tensor t;
            t.name = kv.first;
            t.dtype = v.at("dtype", "tensor field").as_str("dtype");
            const int es = t.dtype == "BF16" ? 2 : (t.dtype == "F32" || t.dtype == "U32") ? 4 : 0;
            if (!es) throw Error("Unsupported safetensors dtype '" + t.dtype + "'.");
            const Json &sh = v.at("shape", "tensor field");
            if (sh.kind != Json::Array || sh.arr.empty() || sh.arr.size() > 8) throw Error("Invalid tensor shape.");
            uint64_t elems = 1;
            for (const Json &d : sh.arr) {
                const int64_t n = d.as_int("a tensor dimension");
                if (n < 1 || n > (1ll << 40)) throw Error("Invalid tensor shape.");
                t.shape.push_back(n);
                elems *= (uint64_t)n;
                if (elems > (1ull << 40)) throw Error("Invalid tensor shape.");
            }
            const Json &off = v.at("data_offsets", "tensor field");
            if (off.kind != Json::Array || off.arr.size() != 2) throw Error("Invalid tensor offsets/byte length.");
            const int64_t a = off.arr[0].as_int("an offset"), b = off.arr[1].as_int("an offset");
            if (a < 0 || b < a || (uint64_t)b > data_bytes || (uint64_t)(b - a) != elems * es)
                throw Error("Invalid tensor offsets/byte length.");
            t.start = data0 + (uint64_t)a;
            t.bytes = (uint64_t)(b - a);
            if (!tensors_.emplace(t.name, t).second) throw Error("Duplicate tensor name.");
            ranges.emplace_back(t.start, t.bytes);
        }
        std::sort(ranges.begin(), ranges.end());
        uint64_t prev = data0;
        for (const auto &r : ranges) {
            if (r.first < prev) throw Error("Overlapping tensors.");
            prev = r.first + r.second;
        }
    }
    // The tensor `name` with exactly `shape` (SafeTensors.Get, SafeTensors.cs:46-51).
    const Tensor &get(const std::string &name, const std::vector<int64_t> &shape) const {
        auto it = tensors_.find(name);
        if (it == tensors_.end() || it->second.shape != shape)
            throw Error("Missing tensor or shape mismatch: " + name + ".");
        return it->second;
    }
    void read(const Tensor &t, void *dst) const {
        FILE *f = std::fopen(path_.c_str(), "rb");
        if (!f) throw Error("Cannot open shard " + path_ + ".");
        const bool ok = fseeko(f, (off_t)t.start, SEEK_SET) == 0 && std::fread(dst, 1, t.bytes, f) == t.bytes;
        std::fclose(f);
        if (!ok) throw Error("Cannot read tensor " + t.name + ".");
    }

private:
    std::string path_;
    std::map<std::string, Tensor> tensors_;
};

// ------------------------------------------------------------------ the MoE block of one layer

// The eight matrices of a layer in di_moe_layer_create order, as the reference names them
// (Qwen36Weights.cs:93-100): router and shared-route gate always 8-bit.
struct MatrixSpec {
    const char *suffix;  // after "language_model.model.layers.{l}."
    int experts_is_E;    // 1: [E, rows, cols]; 0: one expert
    int rows_of, cols_of;  // 0 = E, 1 = D, 2 = I, 3 = one row
    int force8;
};
constexpr MatrixSpec kMatrices[8] = {
    {"mlp.gate", 0, 0, 1, 1},                       // router [E, D]
    {"mlp.switch_mlp.gate_proj", 1, 2, 1, 0},       // [E, I, D]
    {"mlp.switch_mlp.up_proj", 1, 2, 1, 0},         // [E, I, D]
    {"mlp.switch_mlp.down_proj", 1, 1, 2, 0},       // [E, D, I]
    {"mlp.shared_expert.gate_proj", 0, 2, 1, 0},    // [I, D]
    {"mlp.shared_expert.up_proj", 0, 2, 1, 0},      // [I, D]
    {"mlp.shared_expert.down_proj", 0, 1, 2, 0},    // [D, I]
    {"mlp.shared_expert_gate", 0, 3, 1, 1},         // [1, D]
};

struct PlannedMatrix {
    int experts = 1, rows = 0, cols = 0, bits = 8;
    const Shard *shard[3] = {};  // weight, scales, biases
    Tensor t[3];
};

struct LayerPlan {
    int E = 0, D = 0, I = 0, bits = 0;
    PlannedMatrix m[8];
    const Shard *norm_shard = nullptr;
    Tensor norm;  // post_attention_layernorm.weight [D], BF16 or F32
    std::map<std::string, std::unique_ptr<Shard>> shards;
};

// Reads and validates everything the MoE block of `layer` needs, before any upload.
inline void plan_layer(const std::string &dir, int layer, LayerPlan &P) {
    const Json cfg = parse_file(dir + "/config.json");
    const Json *tc = cfg.get("text_config");
    const Json &c = tc ? *tc : cfg;
    P.D = (int)c.at("hidden_size", "config field").as_int("hidden_size");
    P.E = (int)c.at("num_experts", "config field").as_int("num_experts");
    P.I = (int)c.at("moe_intermediate_size", "config field").as_int("moe_intermediate_size");
    const int64_t k = c.at("num_experts_per_tok", "config field").as_int("num_experts_per_tok");
    const int64_t nl = c.at("num_hidden_layers", "config field").as_int("num_hidden_layers");
    if (k != 8) throw Error("Only top-8 routing is implemented.");
    if (const Json *ntp = c.get("norm_topk_prob"))
        if (ntp->kind != Json::Bool || !ntp->b) throw Error("Only renormalised top-k probabilities are implemented.");
    if (layer < 0 || layer >= nl) throw Error("Layer index out of range.");
    if (P.E < 8 || P.E > 256 || P.D < 256 || P.D % 256 || P.I < 64 || P.I % 64)
        throw Error("Unsupported MoE geometry in config.json.");
    const Json &q = cfg.at("quantization", "config field");
    P.bits = (int)q.at("bits", "quantization field").as_int("bits");
    if (q.at("group_size", "quantization field").as_int("group_size") != 64 || (P.bits != 5 && P.bits != 8))
        throw Error("Expected affine 5-bit or 8-bit/group64 weights.");
    if (const Json *mode = q.get("mode"))
        if (mode->as_str("mode") != "affine") throw Error("Expected affine 5-bit or 8-bit/group64 weights.");
    const Json idx = parse_file(dir + "/model.safetensors.index.json");
    const Json &map = idx.at("weight_map", "index field");
    auto shard_for = [&](const std::string &name) -> const Shard * {
        const std::string &file = map.at(name, "tensor in the weight map").as_str("a shard name");
        // Qwen36Weights.cs:62-64: the shard must be a plain file name inside the directory
        if (file.empty() || file == "." || file == ".." || file.find('/') != std::string::npos ||
            file.find('\\') != std::string::npos)
            throw Error("Unsafe shard path.");
        auto it = P.shards.find(file);
        if (it == P.shards.end()) it = P.shards.emplace(file, std::make_unique<Shard>(dir + "/" + file)).first;
        return it->second.get();
    };
    const std::string pre = "language_model.model.layers." + std::to_string(layer) + ".";
    const int dims[4] = {P.E, P.D, P.I, 1};
    for (int i = 0; i < 8; ++i) {
        const MatrixSpec &s = kMatrices[i];
        PlannedMatrix &M = P.m[i];
        const std::string prefix = pre + s.suffix;
        M.bits = s.force8 ? 8 : P.bits;
        // a per-matrix override must agree with the bits the block expects (Qwen36Weights.cs:68-71)
        if (const Json *o = q.get(prefix)) {
            if (o->kind != Json::Object || o->at("bits", "override field").as_int("bits") != M.bits ||
                o->at("group_size", "override field").as_int("group_size") != 64)
                throw Error("Unsupported quantization override: " + prefix);
            if (const Json *mode = o->get("mode"))
                if (mode->as_str("mode") != "affine") throw Error("Unsupported quantization override: " + prefix);
        }
        M.experts = s.experts_is_E ? P.E : 1;
        M.rows = dims[s.rows_of];
        M.cols = dims[s.cols_of];
        if ((int64_t)M.cols * M.bits % 32) throw Error("Unsupported packed row width: " + prefix);
        auto shape = [&](int width) {
            std::vector<int64_t> v;
            if (s.experts_is_E) v.push_back(M.experts);
            v.push_back(M.rows);
            v.push_back(width);
            return v;
        };
        const char *kinds[3] = {".weight", ".scales", ".biases"};
        const int widths[3] = {M.cols * M.bits / 32, M.cols / 64, M.cols / 64};
        const char *dts[3] = {"U32", "BF16", "BF16"};
        for (int j = 0; j < 3; ++j) {
            M.shard[j] = shard_for(prefix + kinds[j]);
            M.t[j] = M.shard[j]->get(prefix + kinds[j], shape(widths[j]));
            if (M.t[j].dtype != dts[j]) throw Error("Expected U32 packed weights and BF16 affine parameters.");
        }
    }
    const std::string nn = pre + "post_attention_layernorm.weight";
    P.norm_shard = shard_for(nn);
    P.norm = P.norm_shard->get(nn, {P.D});
    if (P.norm.dtype != "BF16" && P.norm.dtype != "F32") throw Error("BF16 or F32 norm weights required.");
}

// The norm weights as f32 (bf16 widened by <<16); non-finite values are rejected (SafeTensors.cs:70).
inline std::vector<float> read_norm(const LayerPlan &P) {
    std::vector<float> out((size_t)P.D);
    if (P.norm.dtype == "F32") {
        P.norm_shard->read(P.norm, out.data());
    } else {
        std::vector<uint16_t> h((size_t)P.D);
        P.norm_shard->read(P.norm, h.data());
        for (int i = 0; i < P.D; ++i) {
            const uint32_t u = (uint32_t)h[i] << 16;
            std::memcpy(&out[i], &u, 4);
        }
    }
    for (float v : out)
        if (!(v == v) || v - v != 0.0f) throw Error("Non-finite tensor values.");
    return out;
}

}  // namespace ckpt
}  // namespace di
