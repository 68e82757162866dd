// adai_b200.hpp — header-only C++17 wrapper over the C ABI (adai_b200.h), for the reference's C++
// host code. Errors become the exception types the reference throws on the same conditions
// (std::invalid_argument, std::out_of_range, std::runtime_error), as its CUDA_CHECK / shape
// checks do (src/gpu/GPUUtils.hpp:54-70, src/gpu/MatrixGPU.hpp:513-520, src/KVCache.hpp:99-110).
//
//   adai_b200::Context ctx(/*device=*/0);
//   ctx.upload(desc, tensors);                       // reference setter order, host fp32
//   adai_b200::KVArena kv(ctx, 128, 300, 1024);
//   adai_b200::BatchGenerator gen(kv);
//   auto outs = gen.generate(requests);              // encoder once, stacked greedy decode
#ifndef ADAI_B200_HPP
#define ADAI_B200_HPP

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "adai_b200.h"

namespace adai_b200 {

struct NonFiniteLogits : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct DeviceTimeout : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void check(int rc) {
    if (rc == ADAI_B200_OK) return;
    const std::string msg = adai_b200_last_error();
    switch (rc) {
        case ADAI_B200_ERR_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        case ADAI_B200_ERR_OUT_OF_RANGE: throw std::out_of_range(msg);
        case ADAI_B200_ERR_NONFINITE: throw NonFiniteLogits(msg);
        case ADAI_B200_ERR_TIMEOUT: throw DeviceTimeout(msg);
        default: throw std::runtime_error(msg);
    }
}

// One GPU: the reference GPUManager's device + stream (src/gpu/GPUUtils.hpp:98-530).
class Context {
   public:
    explicit Context(int device = 0, float mem_fraction = 0.f) {
        check(adai_b200_ctx_create(device, mem_fraction, &ctx_));
    }
    ~Context() {
        if (ctx_) adai_b200_ctx_destroy(ctx_);
    }
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;

    // Host fp32 row-major tensors in the order adai_b200_model_upload documents.
    void upload(const adai_b200_model_desc& d, const std::vector<const float*>& tensors,
                const float* pe_table = nullptr) {
        const int n = adai_b200_model_tensor_count(&d);
        if (n != static_cast<int>(tensors.size()))
            throw std::invalid_argument("model needs " + std::to_string(n) + " tensors, got " +
                                        std::to_string(tensors.size()));
        check(adai_b200_model_upload(ctx_, &d, tensors.data(), pe_table));
        desc_ = d;
    }
    // A checkpoint directory in the reference's SafeTensors layout (ModelSerializer,
    // src/ModelSerializer.cpp:243-579); with `expect`, its shape must match.
    void load(const std::string& dir, const adai_b200_model_desc* expect = nullptr) {
        check(adai_b200_model_load(ctx_, dir.c_str(), expect));
        check(adai_b200_checkpoint_config(dir.c_str(), &desc_));
    }
    void synchronize(double timeout_s = 0.0) { check(adai_b200_ctx_synchronize(ctx_, timeout_s)); }
    const adai_b200_model_desc& desc() const { return desc_; }
    adai_b200_ctx* get() const { return ctx_; }

   private:
    adai_b200_ctx* ctx_ = nullptr;
    adai_b200_model_desc desc_{};
};

// Per-sequence self/cross caches of `max_slots` sequences (DecoderKVCache per slot,
// src/KVCache.hpp:155-245; GPUDecoderKVCache's fixed capacity, src/gpu/MatrixGPU.hpp:563-623).
class KVArena {
   public:
    KVArena(Context& ctx, int max_slots, int self_capacity, int cross_capacity) : ctx_(ctx) {
        check(adai_b200_kv_create(ctx.get(), max_slots, self_capacity, cross_capacity, &kv_));
        max_slots_ = max_slots;
    }
    ~KVArena() {
        if (kv_) adai_b200_kv_destroy(ctx_.get(), kv_);
    }
    KVArena(const KVArena&) = delete;
    KVArena& operator=(const KVArena&) = delete;

    void clear(int slot) { check(adai_b200_kv_reset(ctx_.get(), kv_, slot)); }
    void clear_self_attention(int slot) { check(adai_b200_kv_clear_self(ctx_.get(), kv_, slot)); }
    int current_length(int slot) const {
        int s = 0, c = 0;
        check(adai_b200_kv_length(ctx_.get(), kv_, slot, &s, &c));
        return s;
    }
    // LLMEncoder::encode_with_mask for each source + the cross K/V of every decoder layer.
    void encode(const std::vector<int>& slots, const std::vector<std::vector<int>>& sources) {
        std::vector<int> ids, lens;
        for (const auto& s : sources) {
            lens.push_back(static_cast<int>(s.size()));
            ids.insert(ids.end(), s.begin(), s.end());
        }
        check(adai_b200_encode(ctx_.get(), kv_, static_cast<int>(slots.size()), slots.data(),
                               ids.data(), lens.data(), nullptr));
    }
    // One stacked LLMDecoder::forward_with_cache step + LanguageModelHead + first-max argmax.
    std::vector<int> decode_step(const std::vector<int>& slots, const std::vector<int>& ids,
                                 std::vector<float>* logits = nullptr) {
        std::vector<int> next(slots.size());
        if (logits) logits->resize(slots.size() * static_cast<size_t>(ctx_.desc().vocab));
        check(adai_b200_decode_step(ctx_.get(), kv_, static_cast<int>(slots.size()), slots.data(),
                                    ids.data(), next.data(), logits ? logits->data() : nullptr));
        return next;
    }
    int max_slots() const { return max_slots_; }
    adai_b200_kv* get() const { return kv_; }

   private:
    Context& ctx_;
    adai_b200_kv* kv_ = nullptr;
    int max_slots_ = 0;
};

// A generation request: source ids, the number of new tokens at most (TextGenerator's
// max_length, src/TextGenerator.cpp:213-214) and the ids that end it — EOS and PAD, as
// adai::is_stop_token decides (src/SpecialTokens.hpp:162-164).
struct Request {
    std::vector<int> source;
    int max_length = 32;
    int bos = 2;
    std::vector<int> stop_ids = {3, 0};
};

// As generate_greedy returns it (src/TextGenerator.cpp:209-233): the start token, then every
// generated id, the stop id included when one ended the request.
struct Result {
    std::vector<int> tokens;
    std::string error;  // set when this request failed; the other requests are unaffected
};

// BatchedInferenceEngine::process_batch (src/BatchedInferenceEngine.hpp:465-537) with a real
// batch: every request is encoded, then all of them advance together one stacked decode step at a
// time; a request leaves the batch at a stop id or at its max_length. A request that cannot be
// admitted (bad ids, too long) gets its error and the others proceed.
class BatchGenerator {
   public:
    explicit BatchGenerator(KVArena& kv) : kv_(kv) {}

    std::vector<Result> generate(const std::vector<Request>& reqs) {
        std::vector<Result> out(reqs.size());
        for (size_t base = 0; base < reqs.size(); base += static_cast<size_t>(kv_.max_slots())) {
            const size_t end = std::min(reqs.size(), base + static_cast<size_t>(kv_.max_slots()));
            run_wave(reqs, base, end, out);
        }
        return out;
    }

   private:
    void run_wave(const std::vector<Request>& reqs, size_t base, size_t end, std::vector<Result>& out) {
        std::vector<int> slots, feed;
        std::vector<size_t> owner;
        for (size_t i = base; i < end; ++i) {
            const int slot = static_cast<int>(i - base);
            try {
                kv_.encode({slot}, {reqs[i].source});
                out[i].tokens.push_back(reqs[i].bos);
                slots.push_back(slot);
                feed.push_back(reqs[i].bos);
                owner.push_back(i);
            } catch (const std::exception& e) {
                out[i].error = e.what();
            }
        }
        std::vector<int> remaining;
        for (size_t j = 0; j < owner.size(); ++j) remaining.push_back(reqs[owner[j]].max_length);
        for (size_t j = slots.size(); j-- > 0;) {
            if (remaining[j] > 0) continue;
            slots.erase(slots.begin() + static_cast<long>(j));
            feed.erase(feed.begin() + static_cast<long>(j));
            owner.erase(owner.begin() + static_cast<long>(j));
            remaining.erase(remaining.begin() + static_cast<long>(j));
        }
        while (!slots.empty()) {
            const std::vector<int> next = kv_.decode_step(slots, feed);
            std::vector<int> s2, f2, r2;
            std::vector<size_t> o2;
            for (size_t j = 0; j < slots.size(); ++j) {
                const Request& rq = reqs[owner[j]];
                const bool stop = std::find(rq.stop_ids.begin(), rq.stop_ids.end(), next[j]) !=
                                  rq.stop_ids.end();
                out[owner[j]].tokens.push_back(next[j]);
                if (!stop && remaining[j] > 1) {
                    s2.push_back(slots[j]);
                    f2.push_back(next[j]);
                    r2.push_back(remaining[j] - 1);
                    o2.push_back(owner[j]);
                }
            }
            slots.swap(s2);
            feed.swap(f2);
            remaining.swap(r2);
            owner.swap(o2);
        }
    }

    KVArena& kv_;
};

}  // namespace adai_b200

#endif  // ADAI_B200_HPP
