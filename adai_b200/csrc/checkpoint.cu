// checkpoint.cu — SafeTensors checkpoints of the reference's encoder-decoder, read on the host.
//
// The tensor names and layouts follow the reference's exporter (src/ModelSerializer.cpp:243-391):
// T5-style names, projection matrices stored [out, in] (transposed from the reference's
// right-multiplied W[in, out]), vectors and embedding tables as they are. The JSON reader below
// handles the subset a SafeTensors header and config.json use (objects, arrays, strings, numbers,
// true / false / null).
#include "checkpoint.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace adai_b200 {
namespace {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* find(const std::string& key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonReader {
   public:
    JsonReader(const char* p, const char* end, const std::string& what) : p_(p), end_(end), what_(what) {}

    Json document() {
        Json v = value(0);
        ws();
        if (p_ != end_) error("trailing characters");
        return v;
    }

   private:
    const char* p_;
    const char* end_;
    std::string what_;

    [[noreturn]] void error(const char* msg) const {
        throw std::invalid_argument(what_ + ": malformed JSON (" + msg + ")");
    }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool take(char c) {
        ws();
        if (p_ < end_ && *p_ == c) {
            ++p_;
            return true;
        }
        return false;
    }
    void expect(char c) {
        if (!take(c)) error("unexpected character");
    }
    bool literal(const char* s) {
        const size_t n = std::strlen(s);
        if (static_cast<size_t>(end_ - p_) >= n && std::memcmp(p_, s, n) == 0) {
            p_ += n;
            return true;
        }
        return false;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (end_ - p_ < 4) error("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
            else error("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        expect('"');
        std::string out;
        while (true) {
            if (p_ >= end_) error("unterminated string");
            const char c = *p_++;
            if (c == '"') break;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p_ >= end_) error("unterminated escape");
            const char e = *p_++;
            switch (e) {
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
                    if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: error("bad escape");
            }
        }
        return out;
    }
    Json value(int depth) {
        if (depth > 64) error("nesting too deep");
        ws();
        if (p_ >= end_) error("unexpected end");
        Json v;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = Json::Obj;
            if (take('}')) return v;
            do {
                ws();
                std::string k = string();
                expect(':');
                v.obj.emplace_back(std::move(k), value(depth + 1));
            } while (take(','));
            expect('}');
        } else if (c == '[') {
            ++p_;
            v.kind = Json::Arr;
            if (take(']')) return v;
            do v.arr.push_back(value(depth + 1));
            while (take(','));
            expect(']');
        } else if (c == '"') {
            v.kind = Json::Str;
            v.str = string();
        } else if (literal("true")) {
            v.kind = Json::Bool;
            v.b = true;
        } else if (literal("false")) {
            v.kind = Json::Bool;
        } else if (literal("null")) {
            v.kind = Json::Null;
        } else {
            const char* s = p_;
            while (p_ < end_ && (std::strchr("+-.eE", *p_) || (*p_ >= '0' && *p_ <= '9'))) ++p_;
            if (p_ == s) error("unexpected character");
            const std::string num(s, p_);
            char* stop = nullptr;
            v.num = std::strtod(num.c_str(), &stop);
            if (stop != num.c_str() + num.size()) error("bad number");
            v.kind = Json::Num;
        }
        return v;
    }
};

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw CheckpointIoError("cannot open " + path);
    return std::string(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

int config_int(const Json& cfg, const char* key, const std::string& path) {
    const Json* v = cfg.find(key);
    if (!v || v->kind != Json::Num || v->num != static_cast<double>(static_cast<int>(v->num)))
        throw std::invalid_argument(path + ": missing or non-integer \"" + key + "\"");
    return static_cast<int>(v->num);
}

struct TensorEntry {
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte range within the data region
};

class SafeTensors {
   public:
    explicit SafeTensors(const std::string& path) : path_(path), f_(path, std::ios::binary) {
        if (!f_) throw CheckpointIoError("cannot open " + path);
        f_.seekg(0, std::ios::end);
        const uint64_t size = static_cast<uint64_t>(f_.tellg());
        f_.seekg(0);
        uint64_t hlen = 0;
        unsigned char b[8];
        if (size < 8 || !f_.read(reinterpret_cast<char*>(b), 8))
            throw std::invalid_argument(path + ": too short for a SafeTensors header");
        for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];  // little-endian
        if (hlen == 0 || hlen > size - 8 || hlen > (uint64_t(1) << 30))
            throw std::invalid_argument(path + ": invalid SafeTensors header length");
        std::string header(static_cast<size_t>(hlen), '\0');
        if (!f_.read(&header[0], static_cast<std::streamsize>(hlen)))
            throw CheckpointIoError(path + ": cannot read the header");
        data_start_ = 8 + hlen;
        const uint64_t data_size = size - data_start_;
        const Json h = JsonReader(header.data(), header.data() + header.size(), path).document();
        if (h.kind != Json::Obj) throw std::invalid_argument(path + ": header is not a JSON object");
        for (const auto& kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            const Json& e = kv.second;
            const Json* dt = e.find("dtype");
            const Json* sh = e.find("shape");
            const Json* off = e.find("data_offsets");
            if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off ||
                off->kind != Json::Arr || off->arr.size() != 2)
                throw std::invalid_argument(path + ": malformed entry for tensor '" + kv.first + "'");
            TensorEntry t;
            uint64_t elems = 1;
            for (const Json& d : sh->arr) {
                if (d.kind != Json::Num || d.num < 0)
                    throw std::invalid_argument(path + ": bad shape of tensor '" + kv.first + "'");
                t.shape.push_back(static_cast<int64_t>(d.num));
                elems *= static_cast<uint64_t>(d.num);
            }
            t.begin = static_cast<uint64_t>(off->arr[0].num);
            t.end = static_cast<uint64_t>(off->arr[1].num);
            if (t.end < t.begin || t.end > data_size)
                throw std::invalid_argument(path + ": data range of tensor '" + kv.first + "' is outside the file");
            if (dt->str == "F32" && t.end - t.begin != elems * 4)
                throw std::invalid_argument(path + ": size of tensor '" + kv.first + "' does not match its shape");
            dtype_[kv.first] = dt->str;
            entries_[kv.first] = std::move(t);
        }
    }

    bool has(const std::string& name) const { return entries_.count(name) != 0; }

    // Reads tensor `name`, which must be F32 with the given shape, into dst. With transpose, the
    // stored [rows, cols] matrix is written as [cols, rows].
    void read(const std::string& name, const std::vector<int64_t>& shape, float* dst, bool transpose) {
        auto it = entries_.find(name);
        if (it == entries_.end()) throw std::invalid_argument(path_ + ": required tensor missing: " + name);
        if (dtype_[name] != "F32")
            throw std::invalid_argument(path_ + ": tensor '" + name + "' is " + dtype_[name] + ", expected F32");
        if (it->second.shape != shape) {
            std::string want, got;
            for (int64_t s : shape) want += (want.empty() ? "" : ",") + std::to_string(s);
            for (int64_t s : it->second.shape) got += (got.empty() ? "" : ",") + std::to_string(s);
            throw std::invalid_argument(path_ + ": tensor '" + name + "' has shape [" + got + "], expected [" + want + "]");
        }
        const uint64_t n = (it->second.end - it->second.begin) / 4;
        f_.clear();
        f_.seekg(static_cast<std::streamoff>(data_start_ + it->second.begin));
        if (!transpose) {
            if (!f_.read(reinterpret_cast<char*>(dst), static_cast<std::streamsize>(n * 4)))
                throw CheckpointIoError(path_ + ": cannot read tensor '" + name + "'");
            return;
        }
        const size_t rows = static_cast<size_t>(shape[0]), cols = static_cast<size_t>(shape[1]);
        std::vector<float> band;
        const size_t band_rows = 64;  // transpose a band of stored rows at a time
        for (size_t r0 = 0; r0 < rows; r0 += band_rows) {
            const size_t nr = std::min(band_rows, rows - r0);
            band.resize(nr * cols);
            if (!f_.read(reinterpret_cast<char*>(band.data()), static_cast<std::streamsize>(nr * cols * 4)))
                throw CheckpointIoError(path_ + ": cannot read tensor '" + name + "'");
            for (size_t c = 0; c < cols; ++c)
                for (size_t r = 0; r < nr; ++r) dst[c * rows + r0 + r] = band[r * cols + c];
        }
    }

   private:
    std::string path_;
    std::ifstream f_;
    uint64_t data_start_ = 0;
    std::map<std::string, TensorEntry> entries_;
    std::map<std::string, std::string> dtype_;
};

}  // namespace

adai_b200_model_desc read_safetensors_config(const std::string& dir) {
    const std::string path = dir + "/config.json";
    const std::string text = read_file(path);
    const Json cfg = JsonReader(text.data(), text.data() + text.size(), path).document();
    if (cfg.kind != Json::Obj) throw std::invalid_argument(path + ": not a JSON object");
    adai_b200_model_desc d{};
    d.vocab = config_int(cfg, "vocab_size", path);
    d.d_model = config_int(cfg, "d_model", path);
    d.n_heads = config_int(cfg, "num_heads", path);
    d.d_ff = config_int(cfg, "d_ff", path);
    d.enc_layers = config_int(cfg, "num_layers", path);
    d.dec_layers = config_int(cfg, "num_decoder_layers", path);
    d.max_seq = config_int(cfg, "max_length", path);
    return d;
}

std::vector<size_t> upload_tensor_sizes(const adai_b200_model_desc& d) {
    const size_t V = d.vocab, D = d.d_model, F = d.d_ff;
    std::vector<size_t> n;
    n.push_back(V * D);
    for (int i = 0; i < d.enc_layers; ++i)
        for (size_t s : {D, D, D * D, D * D, D * D, D * D, D, D, D * F, F, F * D, D}) n.push_back(s);
    n.push_back(D);
    n.push_back(D);
    n.push_back(V * D);
    for (int i = 0; i < d.dec_layers; ++i)
        for (size_t s : {D, D, D * D, D * D, D * D, D * D, D, D, D * D, D * D, D * D, D * D, D, D,
                         D * F, F, F * D, D})
            n.push_back(s);
    n.push_back(D);
    n.push_back(D);
    n.push_back(D * V);
    n.push_back(V);
    return n;
}

void read_safetensors_tensors(const std::string& dir, const adai_b200_model_desc& d,
                              const std::vector<float*>& out) {
    const std::vector<size_t> sizes = upload_tensor_sizes(d);
    if (out.size() != sizes.size())
        throw std::invalid_argument("need " + std::to_string(sizes.size()) + " output buffers");
    SafeTensors st(dir + "/model.safetensors");
    const int64_t V = d.vocab, D = d.d_model, F = d.d_ff;
    size_t k = 0;
    auto vec = [&](const std::string& name, int64_t n) { st.read(name, {n}, out[k++], false); };
    // [out, in] in the file -> W[in, out]
    auto mat = [&](const std::string& name, int64_t rows, int64_t cols) {
        st.read(name, {rows, cols}, out[k++], true);
    };
    auto norm = [&](const std::string& prefix) {  // optional final LayerNorm
        if (st.has(prefix + ".weight") && st.has(prefix + ".bias")) {
            vec(prefix + ".weight", D);
            vec(prefix + ".bias", D);
        } else {
            for (int j = 0; j < 2; ++j, ++k)
                for (int64_t i = 0; i < D; ++i) out[k][i] = (j == 0) ? 1.f : 0.f;
        }
    };
    st.read("model.shared.weight", {V, D}, out[k++], false);
    for (int i = 0; i < d.enc_layers; ++i) {
        const std::string b = "model.encoder.block." + std::to_string(i);
        vec(b + ".layer.0.layer_norm.weight", D);
        vec(b + ".layer.0.layer_norm.bias", D);
        for (const char* p : {"q", "k", "v", "o"}) mat(b + ".layer.0.SelfAttention." + p + ".weight", D, D);
        vec(b + ".layer.1.layer_norm.weight", D);
        vec(b + ".layer.1.layer_norm.bias", D);
        mat(b + ".layer.1.DenseReluDense.wi.weight", F, D);
        vec(b + ".layer.1.DenseReluDense.wi.bias", F);
        mat(b + ".layer.1.DenseReluDense.wo.weight", D, F);
        vec(b + ".layer.1.DenseReluDense.wo.bias", D);
    }
    norm("model.encoder.final_layer_norm");
    st.read(st.has("model.decoder.embed_tokens.weight") ? "model.decoder.embed_tokens.weight"
                                                        : "model.shared.weight",
            {V, D}, out[k++], false);
    for (int i = 0; i < d.dec_layers; ++i) {
        const std::string b = "model.decoder.block." + std::to_string(i);
        vec(b + ".layer.0.layer_norm.weight", D);
        vec(b + ".layer.0.layer_norm.bias", D);
        for (const char* p : {"q", "k", "v", "o"}) mat(b + ".layer.0.SelfAttention." + p + ".weight", D, D);
        vec(b + ".layer.1.layer_norm.weight", D);
        vec(b + ".layer.1.layer_norm.bias", D);
        for (const char* p : {"q", "k", "v", "o"}) mat(b + ".layer.1.EncDecAttention." + p + ".weight", D, D);
        vec(b + ".layer.2.layer_norm.weight", D);
        vec(b + ".layer.2.layer_norm.bias", D);
        mat(b + ".layer.2.DenseReluDense.wi.weight", F, D);
        vec(b + ".layer.2.DenseReluDense.wi.bias", F);
        mat(b + ".layer.2.DenseReluDense.wo.weight", D, F);
        vec(b + ".layer.2.DenseReluDense.wo.bias", D);
    }
    norm("model.decoder.final_layer_norm");
    mat("lm_head.weight", V, D);
    vec("lm_head.bias", V);
    if (k != sizes.size()) throw std::logic_error("checkpoint tensor order out of step");
}

// ---------------------------------------------------------------------------------------------
// The reference's own checkpoint: EncoderDecoderModel::save_model(P) (src/EncoderDecoderModel.cpp:
// 960-985) writes P.config, P.encoder, P.decoder and P.lm_head, and the encoder and decoder write
// one file per component next to them (src/LLMEncoder.cpp:271-292, src/Decoder.cpp:396-416,
// src/EncoderBlock.cpp:207-229, src/DecoderBlock.cpp:567-621). Every file is a sequence of
// native-endian int32 / float / uint8 values and row-major float matrices with nothing between
// them (adai::binio, src/BinaryIO.cpp); the reference's loaders check each shape and that nothing
// follows the last value.
namespace {

constexpr int32_t kBinaryConfigMarker = -20260721;  // src/EncoderDecoderModel.cpp:128
constexpr int32_t kBinaryConfigVersion = 2;         // :129, pre-LN blocks

struct BinaryConfig {
    adai_b200_model_desc d{};
    int bos = 2, eos = 3, pad = 0;
};

bool file_exists(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    return static_cast<bool>(f);
}

class BinFile {
   public:
    explicit BinFile(const std::string& path) : path_(path), f_(path, std::ios::binary) {
        if (!f_) throw CheckpointIoError("Failed to open file for reading: " + path);
    }
    template <class T>
    T value(const char* what) {
        T v{};
        bytes(&v, sizeof v, what);
        return v;
    }
    void floats(float* dst, size_t n, const char* what) { bytes(dst, n * sizeof(float), what); }
    // Matches an int32 field against the model's value (the reference's dimension checks).
    void expect_int(int want, const char* what) {
        const int got = value<int32_t>(what);
        if (got != want)
            throw std::invalid_argument("Dimension mismatch in " + path_ + ": " + what + " is " +
                                        std::to_string(got) + ", the model has " + std::to_string(want));
    }
    void expect_end() {
        if (f_.peek() != std::char_traits<char>::eof())
            throw std::invalid_argument("Unexpected trailing data in " + path_ +
                                        " (the file doesn't match this model's shapes)");
    }

   private:
    void bytes(void* dst, size_t n, const char* what) {
        f_.read(static_cast<char*>(dst), static_cast<std::streamsize>(n));
        if (static_cast<size_t>(f_.gcount()) != n)
            throw CheckpointIoError("Truncated or unreadable file " + path_ + " (reading " + what + ")");
    }
    std::string path_;
    std::ifstream f_;
};

BinaryConfig read_binary_config(const std::string& prefix) {
    BinFile f(prefix + ".config");
    if (f.value<int32_t>("format marker") != kBinaryConfigMarker)
        throw std::invalid_argument(prefix + ".config: checkpoint format marker missing/invalid "
                                    "(a checkpoint saved before the pre-LN blocks)");
    const int32_t version = f.value<int32_t>("format version");
    if (version < kBinaryConfigVersion)
        throw std::invalid_argument(prefix + ".config: unsupported older checkpoint format_version " +
                                    std::to_string(version));
    BinaryConfig c;
    c.d.vocab = f.value<int32_t>("architecture");
    c.d.d_model = f.value<int32_t>("architecture");
    c.d.enc_layers = f.value<int32_t>("architecture");
    c.d.dec_layers = f.value<int32_t>("architecture");
    c.d.n_heads = f.value<int32_t>("architecture");
    c.d.d_ff = f.value<int32_t>("architecture");
    c.d.max_seq = f.value<int32_t>("architecture");
    c.bos = f.value<int32_t>("architecture");
    c.eos = f.value<int32_t>("architecture");
    c.pad = f.value<int32_t>("architecture");
    f.expect_end();
    return c;
}

// LayerNorm::load_weights (src/LayerNorm.cpp:277-301): dim, epsilon, gamma, beta. The device
// kernels normalise with epsilon 1e-5, the reference's default (src/LayerNorm.hpp:70).
void read_norm_file(const std::string& path, int D, float* g, float* b) {
    BinFile f(path);
    f.expect_int(D, "dim");
    const float eps = f.value<float>("eps");
    if (!(eps > 0.0f) || !std::isfinite(eps))
        throw std::invalid_argument(path + ": epsilon " + std::to_string(eps) +
                                    " is not a positive finite number");
    if (eps != 1e-5f)
        throw std::invalid_argument(path + ": LayerNorm epsilon " + std::to_string(eps) +
                                    " differs from the 1e-5 the device kernels use");
    f.floats(g, D, "gamma");
    f.floats(b, D, "beta");
    f.expect_end();
}

// TokenEmbedding::load_pretrained (src/TokenEmbedding.cpp:158-178).
void read_embedding_file(const std::string& path, int V, int D, float* out) {
    BinFile f(path);
    f.expect_int(V, "vocab_size");
    f.expect_int(D, "d_model");
    f.floats(out, static_cast<size_t>(V) * D, "embedding matrix");
    f.expect_end();
}

// MultiHeadAttention::load_weights (src/MultiHeadAttention.cpp:682-708).
void read_attention_file(const std::string& path, int D, int H, float* const* w) {
    BinFile f(path);
    f.expect_int(D, "d_model");
    f.expect_int(H, "num_heads");
    for (int i = 0; i < 4; ++i) f.floats(w[i], static_cast<size_t>(D) * D, "W_q / W_k / W_v / W_o");
    f.expect_end();
}

// CrossAttention::load (src/CrossAttention.cpp:811-836).
void read_cross_attention_file(const std::string& path, int D, int H, float* const* w) {
    BinFile f(path);
    f.expect_int(D, "d_model");
    f.expect_int(H, "num_heads");
    f.value<float>("learning_rate");
    for (int i = 0; i < 4; ++i) f.floats(w[i], static_cast<size_t>(D) * D, "W_q / W_k / W_v / W_o");
    f.expect_end();
}

// FeedForward::load_weights (src/FeedForward.cpp:296-320): W1 [D,F], W2 [F,D], b1, b2 — stored in
// that order; the upload order is W1 b1 W2 b2.
void read_ffn_file(const std::string& path, int D, int F, float* w1, float* b1, float* w2, float* b2) {
    BinFile f(path);
    f.expect_int(D, "d_model");
    f.expect_int(F, "d_ff");
    f.floats(w1, static_cast<size_t>(D) * F, "W1");
    f.floats(w2, static_cast<size_t>(F) * D, "W2");
    f.floats(b1, F, "b1");
    f.floats(b2, D, "b2");
    f.expect_end();
}

// LLMEncoder / LLMDecoder header: vocab, d_model, layers, heads, d_ff, max_seq_length (which the
// reference does not check: no weight depends on it).
void read_stack_header(const std::string& path, const adai_b200_model_desc& d, int layers) {
    BinFile f(path);
    f.expect_int(d.vocab, "vocab_size");
    f.expect_int(d.d_model, "d_model");
    f.expect_int(layers, "num_layers");
    f.expect_int(d.n_heads, "num_heads");
    f.expect_int(d.d_ff, "d_ff");
    f.value<int32_t>("max_seq_length");
    f.expect_end();
}

std::string strip_ext(const std::string& p) { return p.substr(0, p.find_last_of('.')); }

void read_binary_tensors(const std::string& prefix, const adai_b200_model_desc& d,
                         const std::vector<float*>& out) {
    const int V = d.vocab, D = d.d_model, H = d.n_heads, F = d.d_ff;
    size_t k = 0;
    // encoder (src/LLMEncoder.cpp:296-350); base strips ".encoder"
    read_stack_header(prefix + ".encoder", d, d.enc_layers);
    const std::string base = strip_ext(prefix + ".encoder");
    // pre-TD-538 checkpoints hold only the shared names (the decoder's copies), which the
    // reference then loads for the encoder too
    auto enc_part = [&](const std::string& name) {
        const std::string cur = base + "_encoder_" + name;
        return file_exists(cur) ? cur : base + "_" + name;
    };
    read_embedding_file(enc_part("token_emb.bin"), V, D, out[k++]);
    for (int i = 0; i < d.enc_layers; ++i) {
        const std::string blk = base + "_encoder_block_" + std::to_string(i) + ".bin";
        {  // EncoderBlock::load_weights (src/EncoderBlock.cpp:231-259)
            BinFile f(blk);
            f.expect_int(D, "d_model");
            f.expect_int(H, "num_heads");
            f.expect_int(F, "d_ff");
            f.value<float>("dropout_rate");
            f.floats(out[k], D, "norm1 gamma");
            f.floats(out[k + 1], D, "norm1 beta");
            f.floats(out[k + 6], D, "norm2 gamma");
            f.floats(out[k + 7], D, "norm2 beta");
            f.expect_end();
        }
        const std::string bb = strip_ext(blk);
        read_attention_file(bb + "_attention.bin", D, H, &out[k + 2]);
        read_ffn_file(bb + "_feedforward.bin", D, F, out[k + 8], out[k + 9], out[k + 10], out[k + 11]);
        k += 12;
    }
    read_norm_file(enc_part("final_norm.bin"), D, out[k], out[k + 1]);
    k += 2;
    // decoder (src/Decoder.cpp:418-452)
    read_stack_header(prefix + ".decoder", d, d.dec_layers);
    const std::string dbase = strip_ext(prefix + ".decoder");
    read_embedding_file(dbase + "_token_emb.bin", V, D, out[k++]);
    for (int i = 0; i < d.dec_layers; ++i) {
        const std::string blk = dbase + "_decoder_block_" + std::to_string(i) + ".bin";
        {  // DecoderBlock::load (src/DecoderBlock.cpp:623-689)
            BinFile f(blk);
            f.expect_int(D, "d_model");
            f.expect_int(H, "num_heads");
            f.expect_int(F, "d_ff");
            f.value<float>("dropout_rate");
            f.value<float>("learning_rate");
            f.floats(out[k], D, "norm1 gamma");
            f.floats(out[k + 1], D, "norm1 beta");
            f.floats(out[k + 6], D, "norm2 gamma");
            f.floats(out[k + 7], D, "norm2 beta");
            f.floats(out[k + 12], D, "norm3 gamma");
            f.floats(out[k + 13], D, "norm3 beta");
            for (const char* what : {"world-model flag", "hippocampal flag"}) {
                if (f.value<uint8_t>(what) != 0)
                    throw std::invalid_argument(
                        blk + ": the block has a gated " +
                        std::string(what).substr(0, std::string(what).size() - 5) +
                        " cross-attention path, which the device decode step does not run");
            }
            f.expect_end();
        }
        read_attention_file(blk + ".self_attn", D, H, &out[k + 2]);
        read_cross_attention_file(blk + ".cross_attn", D, H, &out[k + 8]);
        read_ffn_file(blk + ".ff", D, F, out[k + 14], out[k + 15], out[k + 16], out[k + 17]);
        k += 18;
    }
    read_norm_file(dbase + "_final_norm.bin", D, out[k], out[k + 1]);
    k += 2;
    {  // LanguageModelHead::load (src/LanguageModelHead.cpp:128-143)
        BinFile f(prefix + ".lm_head");
        f.expect_int(D, "d_model");
        f.expect_int(V, "vocab_size");
        f.floats(out[k++], static_cast<size_t>(D) * V, "W_output");
        f.floats(out[k++], V, "bias");
        f.expect_end();
    }
    if (k != out.size()) throw std::logic_error("binary checkpoint tensor order out of step");
}

bool is_safetensors_dir(const std::string& path) { return file_exists(path + "/config.json"); }

void require_checkpoint(const std::string& path) {
    if (!is_safetensors_dir(path) && !file_exists(path + ".config"))
        throw CheckpointIoError("no checkpoint at " + path + " (neither " + path +
                                "/config.json nor " + path + ".config)");
}

}  // namespace

adai_b200_model_desc read_checkpoint_config(const std::string& path) {
    require_checkpoint(path);
    return is_safetensors_dir(path) ? read_safetensors_config(path) : read_binary_config(path).d;
}

void read_checkpoint_tensors(const std::string& path, const adai_b200_model_desc& d,
                             const std::vector<float*>& out) {
    require_checkpoint(path);
    if (out.size() != upload_tensor_sizes(d).size())
        throw std::invalid_argument("need " + std::to_string(upload_tensor_sizes(d).size()) +
                                    " output buffers");
    if (is_safetensors_dir(path)) {
        read_safetensors_tensors(path, d, out);
        return;
    }
    const BinaryConfig c = read_binary_config(path);
    if (std::memcmp(&c.d, &d, sizeof d) != 0)
        throw std::invalid_argument("Model architecture mismatch between " + path +
                                    ".config and the requested model");
    read_binary_tensors(path, d, out);
}

void read_checkpoint_special_tokens(const std::string& path, int* bos, int* eos, int* pad) {
    require_checkpoint(path);
    if (is_safetensors_dir(path)) {
        const std::string cfg_path = path + "/config.json";
        const std::string text = read_file(cfg_path);
        const Json cfg = JsonReader(text.data(), text.data() + text.size(), cfg_path).document();
        *bos = config_int(cfg, "decoder_start_token_id", cfg_path);
        *eos = config_int(cfg, "eos_token_id", cfg_path);
        *pad = config_int(cfg, "pad_token_id", cfg_path);
        return;
    }
    const BinaryConfig c = read_binary_config(path);
    *bos = c.bos;
    *eos = c.eos;
    *pad = c.pad;
}

}  // namespace adai_b200
