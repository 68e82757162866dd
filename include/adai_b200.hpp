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
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
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
    // "<seq> <phase> <kernel>" of the last GPU work queued (describe_last_gpu_work).
    std::string last_work() const {
        char buf[256];
        check(adai_b200_ctx_last_work(ctx_, buf, static_cast<int>(sizeof(buf)), nullptr));
        return buf;
    }
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
    // Per-slot sampling (TextGenerator::generate's rules, adai_b200_kv_set_sampling); nullptr
    // returns the slot to the fused argmax.
    void set_sampling(int slot, const adai_b200_sampling* cfg, const std::vector<int>& history = {}) {
        check(adai_b200_kv_set_sampling(ctx_.get(), kv_, slot, cfg,
                                        history.empty() ? nullptr : history.data(),
                                        static_cast<int>(history.size())));
    }
    int max_slots() const { return max_slots_; }
    adai_b200_kv* get() const { return kv_; }

   private:
    Context& ctx_;
    adai_b200_kv* kv_ = nullptr;
    int max_slots_ = 0;
};

// A generation request: source ids, the number of new tokens at most (TextGenerator's
// max_length, src/TextGenerator.cpp:213-214), the ids that end it — EOS and PAD, as
// adai::is_stop_token decides (src/SpecialTokens.hpp:162-164) — and, optionally, its sampling
// configuration (InferenceRequest::gen_config, src/BatchedInferenceEngine.hpp:120) with its own
// generator seed; without one the request is greedy.
struct Request {
    std::vector<int> source;
    int max_length = 32;
    int bos = 2;
    std::vector<int> stop_ids = {3, 0};
    std::optional<adai_b200_sampling> sampling;
};

// As TextGenerator::generate returns it (src/TextGenerator.cpp:519-565): the start token, then
// every generated id, the stop id included when one ended the request.
struct Result {
    std::vector<int> tokens;
    std::string error;  // set when this request failed; the other requests are unaffected
};

// BatchedInferenceEngine::process_batch (src/BatchedInferenceEngine.hpp:465-537) with a real
// batch and continuous admission (the engine's v2 plan: admit and retire sequences between decode
// steps). Up to max_slots requests decode together, one stacked step at a time. A request leaves
// at a stop id or at its max_length, and its slot goes to the next waiting request before the next
// step. A request that cannot be admitted (bad ids, source too long, a rejected sampling
// configuration) gets its error, and the others proceed. Each request samples from its own
// generator, so its tokens do not depend on the requests around it (the reference engine shares
// one generator among all requests, src/BatchedInferenceEngine.hpp:214-217); the batch size only
// changes how the GEMMs split their sums, which moves logits by float rounding.
class BatchGenerator {
   public:
    explicit BatchGenerator(KVArena& kv) : kv_(kv) {}

    std::vector<Result> generate(const std::vector<Request>& reqs) {
        std::vector<Result> out(reqs.size());
        std::vector<int> free_slots;
        for (int s = kv_.max_slots() - 1; s >= 0; --s) free_slots.push_back(s);
        Active act;
        size_t next = 0;
        admit(reqs, out, next, free_slots, act);
        while (!act.slots.empty()) {
            const std::vector<int> ids = kv_.decode_step(act.slots, act.feed);
            Active keep;
            for (size_t j = 0; j < act.slots.size(); ++j) {
                const Request& rq = reqs[act.owner[j]];
                const bool stop = std::find(rq.stop_ids.begin(), rq.stop_ids.end(), ids[j]) !=
                                  rq.stop_ids.end();
                out[act.owner[j]].tokens.push_back(ids[j]);
                if (!stop && act.remaining[j] > 1)
                    keep.add(act.slots[j], ids[j], act.remaining[j] - 1, act.owner[j]);
                else
                    free_slots.push_back(act.slots[j]);
            }
            act = std::move(keep);
            admit(reqs, out, next, free_slots, act);
        }
        return out;
    }

   private:
    struct Active {
        std::vector<int> slots, feed, remaining;
        std::vector<size_t> owner;
        void add(int slot, int id, int left, size_t who) {
            slots.push_back(slot);
            feed.push_back(id);
            remaining.push_back(left);
            owner.push_back(who);
        }
    };

    // Encodes waiting requests into free slots: all of them in one call, or one by one when the
    // joint call fails, so that a bad request does not hold up the others.
    void admit(const std::vector<Request>& reqs, std::vector<Result>& out, size_t& next,
               std::vector<int>& free_slots, Active& act) {
        std::vector<int> slots;
        std::vector<size_t> who;
        while (!free_slots.empty() && next < reqs.size()) {
            slots.push_back(free_slots.back());
            free_slots.pop_back();
            who.push_back(next++);
        }
        if (slots.empty()) return;
        std::vector<std::vector<int>> sources;
        for (size_t i : who) sources.push_back(reqs[i].source);
        std::vector<bool> ok(slots.size(), true);
        try {
            kv_.encode(slots, sources);
        } catch (const std::exception&) {
            for (size_t j = 0; j < slots.size(); ++j) {
                try {
                    kv_.encode({slots[j]}, {sources[j]});
                } catch (const std::exception& e) {
                    out[who[j]].error = e.what();
                    ok[j] = false;
                }
            }
        }
        for (size_t j = 0; j < slots.size(); ++j) {
            if (!ok[j]) continue;
            const Request& rq = reqs[who[j]];
            try {  // the slot's previous occupant may have sampled: always (re)configure
                kv_.set_sampling(slots[j], rq.sampling ? &*rq.sampling : nullptr);
            } catch (const std::exception& e) {
                out[who[j]].error = e.what();
                ok[j] = false;
            }
        }
        for (size_t j = 0; j < slots.size(); ++j) {
            const Request& rq = reqs[who[j]];
            if (ok[j]) out[who[j]].tokens.push_back(rq.bos);
            if (ok[j] && rq.max_length > 0)
                act.add(slots[j], rq.bos, rq.max_length, who[j]);
            else
                free_slots.push_back(slots[j]);
        }
    }

    KVArena& kv_;
};

}  // namespace adai_b200

#endif  // ADAI_B200_HPP
