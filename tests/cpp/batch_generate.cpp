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
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <typeinfo>

#include "adai_b200.hpp"

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
