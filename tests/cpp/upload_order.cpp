// Reference-side check of include/adai_b200_reference.hpp, built against the reference's own
// sources (oracle/Makefile, target `binding`). It builds the reference's LLMEncoder, LLMDecoder and
// LanguageModelHead with their own random initialisation, walks them with
// adai_b200::tensors_in_upload_order, and writes the tensors together with the reference's own
// greedy decode of one source (encode_with_mask, forward_with_cache per token, the head, first
// maximum), so that a test can replay the tensors through the oracle in upload order and compare.
//
// Usage: upload_order OUT V D H F LE LD MAX_SEQ STEPS id id ...   (the source ids)
// OUT (little-endian): int32 n_tensors; per tensor int64 count + float32[count]; int32 steps;
// int32 ids[steps]; float32 logits[steps][V].
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "KVCache.hpp"
#include "adai_b200_reference.hpp"

int main(int argc, char** argv) {
    if (argc < 11) {
        std::cerr << "usage: upload_order OUT V D H F LE LD MAX_SEQ STEPS ids...\n";
        return 2;
    }
    const int V = std::atoi(argv[2]), D = std::atoi(argv[3]), H = std::atoi(argv[4]);
    const int F = std::atoi(argv[5]), Le = std::atoi(argv[6]), L = std::atoi(argv[7]);
    const int max_seq = std::atoi(argv[8]), steps = std::atoi(argv[9]);
    std::vector<int> src;
    for (int i = 10; i < argc; ++i) src.push_back(std::atoi(argv[i]));

    LLMEncoder enc(V, D, Le, H, F, max_seq);
    LLMDecoder dec(V, D, L, H, F, max_seq, 0);
    LanguageModelHead head(D, V);
    std::vector<std::vector<float>> keep;
    const std::vector<const float*> t = adai_b200::tensors_in_upload_order(enc, dec, head, keep);

    std::ofstream f(argv[1], std::ios::binary);
    const int n = static_cast<int>(t.size());
    f.write(reinterpret_cast<const char*>(&n), 4);
    for (size_t i = 0; i < t.size(); ++i) {
        const long long c = static_cast<long long>(keep[i].size());
        f.write(reinterpret_cast<const char*>(&c), 8);
        f.write(reinterpret_cast<const char*>(t[i]), static_cast<std::streamsize>(c * 4));
    }

    const int S = static_cast<int>(src.size());
    Matrix mask(S, S);
    for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
    Matrix enc_out = enc.encode_with_mask(src, mask);
    DecoderKVCache cache(L);
    std::vector<int> ids;
    std::vector<float> logits;
    int tok = 2;  // BOS
    for (int s = 0; s < steps; ++s) {
        Matrix x = dec.forward_with_cache({tok}, cache, &enc_out, true);
        Matrix lg = head.forward(x);
        const std::vector<float>& row = lg.data[lg.rows - 1];
        tok = static_cast<int>(std::max_element(row.begin(), row.end()) - row.begin());
        ids.push_back(tok);
        logits.insert(logits.end(), row.begin(), row.end());
    }
    f.write(reinterpret_cast<const char*>(&steps), 4);
    f.write(reinterpret_cast<const char*>(ids.data()), static_cast<std::streamsize>(ids.size() * 4));
    f.write(reinterpret_cast<const char*>(logits.data()),
            static_cast<std::streamsize>(logits.size() * 4));
    return f ? 0 : 1;
}
