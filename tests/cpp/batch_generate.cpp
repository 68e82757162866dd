// Drives adai_b200::BatchGenerator (include/adai_b200.hpp) from a binary request file, the way a
// C++ host of the reference would: model tensors in upload order, then greedy requests.
//
// Input (little-endian): int32 vocab, d_model, n_heads, d_ff, enc_layers, dec_layers, max_seq,
// n_tensors; per tensor int64 count + float32[count]; int32 slots, n_requests; per request int32
// max_length, int32 src_len, int32[src_len] ids, int32 sampled, and when sampled is 1 the
// adai_b200_sampling fields in order (float temperature, int32 top_k, float top_p, float
// repetition_penalty, int32 min_length, int32 eos, int32 pad, uint32 seed). Output: one line per
// request, "i: id id ..." or
// "i: error: <message>". With no arguments it only checks that a context can be created and
// prints the exception that refused it ("no-device: <type>: <message>").
//
// With a second argument "engine" the same requests go through adai_b200::BatchedInferenceEngine
// (include/adai_b200_engine.hpp), submitted from three threads at once with a test tokenizer whose
// text is the ids themselves; each line is then "i: <decoded text>" (special ids 0-3 skipped) or
// "i: error: <message>". A request whose source is the single id -1 is submitted with decoder seed
// text instead (the engine must fail that request alone).
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <future>
#include <iostream>
#include <sstream>
#include <thread>
#include <typeinfo>

#include "adai_b200.hpp"
#include "adai_b200_engine.hpp"

// The fields of TextGenerator::GenerationConfig (src/TextGenerator.hpp:65-82) the engine reads.
struct GenConfig {
    int max_length = 100;
    float temperature = 1.0f;
    int top_k = 0;
    float top_p = 1.0f;
    float repetition_penalty = 1.0f;
    int num_beams = 1;
    int min_length = 0;
    int pad_token_id = 0;
    int bos_token_id = 2;
    int eos_token_id = 3;
};

// Text is the ids separated by spaces; decode(..., true) drops the special ids 0-3.
struct IdTokenizer {
    std::vector<int> encode(const std::string& text, bool) const {
        std::istringstream in(text);
        std::vector<int> out;
        for (int v; in >> v;) out.push_back(v);
        return out;
    }
    std::string decode(const std::vector<int>& ids, bool skip_special) const {
        std::string out;
        for (int v : ids) {
            if (skip_special && v >= 0 && v < 4) continue;
            if (!out.empty()) out += ' ';
            out += std::to_string(v);
        }
        return out;
    }
};

static int run_engine(adai_b200::KVArena& kv, const std::vector<adai_b200::Request>& reqs) {
    adai_b200::EngineConfig ec;
    ec.max_batch_size = 4;
    ec.timeout_ms = 20;
    adai_b200::BatchedInferenceEngine<IdTokenizer, GenConfig> engine(
        kv, std::make_shared<IdTokenizer>(), ec, GenConfig(), 7);
    std::vector<std::future<std::string>> futs(reqs.size());
    std::vector<std::thread> th;
    for (int t = 0; t < 3; ++t)
        th.emplace_back([&, t] {
            for (size_t i = t; i < reqs.size(); i += 3) {
                GenConfig g;
                g.max_length = reqs[i].max_length;
                g.temperature = 0.0f;  // greedy
                const bool seed_text = reqs[i].source.size() == 1 && reqs[i].source[0] == -1;
                futs[i] = engine.submit(seed_text ? std::string("5 6") : std::string(), &g,
                                        seed_text ? std::vector<int>{4} : reqs[i].source);
            }
        });
    for (auto& x : th) x.join();
    for (size_t i = 0; i < futs.size(); ++i) {
        try {
            const std::string text = futs[i].get();
            std::cout << i << ": " << text << "\n";
        } catch (const std::exception& e) {
            std::cout << i << ": error: " << e.what() << "\n";
        }
    }
    engine.shutdown();
    bool refused = false;
    try {
        engine.submit("", nullptr, {4});
    } catch (const std::runtime_error&) {
        refused = true;
    }
    const adai_b200::EngineStats st = engine.get_stats();
    std::cout << "stats: requests " << st.total_requests << " batches " << st.total_batches
              << " refused_after_shutdown " << refused << "\n";
    return 0;
}

template <class T>
static T rd(std::ifstream& f) {
    T v{};
    f.read(reinterpret_cast<char*>(&v), sizeof(T));
    if (!f) throw std::runtime_error("truncated input");
    return v;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        try {
            adai_b200::Context ctx(0);
            std::cout << "device-ok\n";
        } catch (const std::runtime_error& e) {
            std::cout << "no-device: runtime_error: " << e.what() << "\n";
        }
        return 0;
    }
    std::ifstream f(argv[1], std::ios::binary);
    adai_b200_model_desc d{};
    d.vocab = rd<int>(f);
    d.d_model = rd<int>(f);
    d.n_heads = rd<int>(f);
    d.d_ff = rd<int>(f);
    d.enc_layers = rd<int>(f);
    d.dec_layers = rd<int>(f);
    d.max_seq = rd<int>(f);
    const int nt = rd<int>(f);
    std::vector<std::vector<float>> store(static_cast<size_t>(nt));
    std::vector<const float*> ptrs;
    for (auto& t : store) {
        t.resize(static_cast<size_t>(rd<long long>(f)));
        f.read(reinterpret_cast<char*>(t.data()), static_cast<std::streamsize>(t.size() * 4));
        ptrs.push_back(t.data());
    }
    const int slots = rd<int>(f);
    std::vector<adai_b200::Request> reqs(static_cast<size_t>(rd<int>(f)));
    for (auto& r : reqs) {
        r.max_length = rd<int>(f);
        r.source.resize(static_cast<size_t>(rd<int>(f)));
        f.read(reinterpret_cast<char*>(r.source.data()), static_cast<std::streamsize>(r.source.size() * 4));
        if (rd<int>(f)) {
            adai_b200_sampling s{};
            s.temperature = rd<float>(f);
            s.top_k = rd<int>(f);
            s.top_p = rd<float>(f);
            s.repetition_penalty = rd<float>(f);
            s.min_length = rd<int>(f);
            s.eos_token_id = rd<int>(f);
            s.pad_token_id = rd<int>(f);
            s.seed = rd<unsigned>(f);
            r.sampling = s;
        }
    }
    adai_b200::Context ctx(0);
    ctx.upload(d, ptrs);
    int longest = 1;
    for (const auto& r : reqs) longest = std::max(longest, r.max_length);
    adai_b200::KVArena kv(ctx, slots, longest, d.max_seq);
    if (argc > 2 && std::string(argv[2]) == "engine") return run_engine(kv, reqs);
    adai_b200::BatchGenerator gen(kv);
    const auto res = gen.generate(reqs);
    for (size_t i = 0; i < res.size(); ++i) {
        std::cout << i << ":";
        if (!res[i].error.empty()) {
            std::cout << " error: " << res[i].error << "\n";
            continue;
        }
        for (int t : res[i].tokens) std::cout << " " << t;
        std::cout << "\n";
    }
    return 0;
}
