// checkpoint.cu — SafeTensors checkpoints of the reference's encoder-decoder, read on the host.
//
// The tensor names and layouts follow the reference's exporter (src/ModelSerializer.cpp:243-391):
// T5-style names, projection matrices stored [out, in] (transposed from the reference's
// right-multiplied W[in, out]), vectors and embedding tables as they are. The JSON reader below
// handles the subset a SafeTensors header and config.json use (objects, arrays, strings, numbers,
// true / false / null).
#include "checkpoint.h"

#include <algorithm>
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

adai_b200_model_desc read_checkpoint_config(const std::string& dir) {
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

void read_checkpoint_tensors(const std::string& dir, const adai_b200_model_desc& d,
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

}  // namespace adai_b200
