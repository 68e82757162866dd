// adai_b200_engine.hpp — the reference's asynchronous serving front end,
// BatchedInferenceEngine::submit(prompt, gen_config*, model_fn) -> std::future<std::string>
// (src/BatchedInferenceEngine.hpp:242-272), over the device decode step. Header-only C++17 on top
// of adai_b200.hpp.
//
// Same contract as the reference engine: submit() queues a request and returns a future; one
// worker thread collects up to max_batch_size queued requests, waiting at most timeout_ms
// (collect_batch, :378-420), and answers each future with the generated text decoded without
// special tokens (TextGenerator::generate_text, src/TextGenerator.cpp:568-581). A full queue or a
// shut-down engine makes submit() throw std::runtime_error with the reference's messages;
// shutdown() answers every request already accepted (TD-212); a request that fails gets its own
// exception and the others go on (process_batch, :465-537).
//
// What differs, and why:
// * The batch really is one batch: the collected requests decode together in stacked device steps
//   (BatchGenerator, continuous admission into freed slots), where the reference generates them
//   one after another (its TD-211).
// * The third argument is the request's encoder input (token ids). The reference takes a
//   per-request ModelForwardFn with that input baked into a host closure (ChatbotAPI passes
//   `[..., input_tokens](decoder_tokens) { return model_->next_token_logits(input_tokens, ...); }`,
//   src/ChatbotAPI.cpp:1086-1091); the device runs the whole model itself, so it needs the ids, not
//   a closure. That call site becomes `submit("", &gen_config, input_tokens)`.
// * The decoder starts at BOS, as ChatbotAPI's batched path does (it submits an empty prompt). A
//   non-empty prompt (decoder seed text) fails that request with std::invalid_argument, and so
//   does num_beams > 1 (beam search recomputes without a cache in the reference).
// * Sampling: each request draws from its own std::mt19937, seeded with seed + its submission
//   number (seed 0: std::random_device), so a request's tokens do not depend on its neighbours;
//   the reference shares one generator among all requests (its TD-214).
//
// Tokenizer: a type with encode(const std::string&, bool) and decode(const std::vector<int>&, bool)
// (BPETokenizer). GenerationConfig: a type with the fields of TextGenerator::GenerationConfig
// (src/TextGenerator.hpp:65-82): max_length, temperature, top_k, top_p, repetition_penalty,
// num_beams, min_length, pad_token_id, bos_token_id, eos_token_id.
#ifndef ADAI_B200_ENGINE_HPP
#define ADAI_B200_ENGINE_HPP

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <exception>
#include <future>
#include <memory>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "adai_b200.hpp"

namespace adai_b200 {

// The fields of BatchedInferenceConfig (src/BatchedInferenceEngine.hpp:49-60) the engine reads.
struct EngineConfig {
    size_t max_batch_size = 32;  // requests per collected batch (also bounded by the arena's slots)
    int timeout_ms = 50;         // longest wait while collecting a batch
    size_t max_queue_size = 1000;
};

// BatchedInferenceStats' counters (src/BatchedInferenceEngine.hpp:69-83).
struct EngineStats {
    uint64_t total_requests = 0;
    uint64_t total_batches = 0;
    uint64_t total_tokens_processed = 0;  // generated ids, start token excluded
    uint64_t requests_timeout = 0;        // batches flushed by the timeout
    uint64_t requests_batch_full = 0;     // batches flushed by the size limit
};

template <class Tokenizer, class GenerationConfig>
class BatchedInferenceEngine {
   public:
    BatchedInferenceEngine(KVArena& kv, std::shared_ptr<Tokenizer> tokenizer,
                           const EngineConfig& config = EngineConfig(),
                           const GenerationConfig& gen_config = GenerationConfig(),
                           uint32_t seed = 0)
        : kv_(kv),
          tokenizer_(std::move(tokenizer)),
          config_(config),
          default_gen_config_(gen_config),
          seed_(seed),
          running_(true) {
        if (!tokenizer_) throw std::invalid_argument("BatchedInferenceEngine: null tokenizer");
        worker_ = std::thread(&BatchedInferenceEngine::loop, this);
    }
    ~BatchedInferenceEngine() { shutdown(); }
    BatchedInferenceEngine(const BatchedInferenceEngine&) = delete;
    BatchedInferenceEngine& operator=(const BatchedInferenceEngine&) = delete;

    std::future<std::string> submit(const std::string& prompt,
                                    const GenerationConfig* gen_config = nullptr,
                                    std::vector<int> encoder_input = {}) {
        Pending p;
        p.prompt = prompt;
        p.gen = gen_config ? *gen_config : default_gen_config_;
        p.source = std::move(encoder_input);
        std::future<std::string> fut = p.result.get_future();
        {
            std::unique_lock<std::mutex> lock(mu_);
            if (!running_) throw std::runtime_error("Cannot submit request: engine is shutdown");
            if (queue_.size() >= config_.max_queue_size)
                throw std::runtime_error("Request queue is full");
            p.number = submitted_++;
            queue_.push(std::move(p));
        }
        cv_.notify_one();
        return fut;
    }

    std::vector<std::future<std::string>> submit_batch(
        const std::vector<std::string>& prompts, const GenerationConfig* gen_config = nullptr,
        const std::vector<std::vector<int>>& encoder_inputs = {}) {
        std::vector<std::future<std::string>> out;
        out.reserve(prompts.size());
        for (size_t i = 0; i < prompts.size(); ++i)
            out.push_back(submit(prompts[i], gen_config,
                                 i < encoder_inputs.size() ? encoder_inputs[i] : std::vector<int>{}));
        return out;
    }

    EngineStats get_stats() const {
        std::lock_guard<std::mutex> lock(stats_mu_);
        return stats_;
    }
    size_t queue_size() const {
        std::lock_guard<std::mutex> lock(mu_);
        return queue_.size();
    }
    bool is_running() const { return running_; }

    // Stops accepting requests and returns once every accepted request has its answer.
    void shutdown() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            if (!running_.exchange(false)) return;
        }
        cv_.notify_all();
        if (worker_.joinable()) worker_.join();
    }

   private:
    struct Pending {
        std::string prompt;
        GenerationConfig gen;
        std::vector<int> source;
        std::promise<std::string> result;
        uint64_t number = 0;
    };

    void loop() {
        while (running_) {
            std::vector<Pending> batch = collect(true);
            if (!batch.empty()) process(batch);
        }
        for (std::vector<Pending> b = collect(false); !b.empty(); b = collect(false)) process(b);
    }

    size_t batch_limit() const {
        const size_t slots = static_cast<size_t>(kv_.max_slots());
        return std::max<size_t>(1, std::min(config_.max_batch_size, slots));
    }

    std::vector<Pending> collect(bool wait) {
        std::vector<Pending> batch;
        std::unique_lock<std::mutex> lock(mu_);
        const size_t limit = batch_limit();
        if (!wait) {
            while (!queue_.empty() && batch.size() < limit) {
                batch.push_back(std::move(queue_.front()));
                queue_.pop();
            }
            return batch;
        }
        const auto deadline =
            std::chrono::steady_clock::now() + std::chrono::milliseconds(config_.timeout_ms);
        while (batch.size() < limit && running_) {
            if (cv_.wait_until(lock, deadline, [this] { return !queue_.empty() || !running_; })) {
                if (!running_) break;
                batch.push_back(std::move(queue_.front()));
                queue_.pop();
                if (batch.size() >= limit) {
                    std::lock_guard<std::mutex> s(stats_mu_);
                    stats_.requests_batch_full++;
                }
            } else {
                if (!batch.empty()) {
                    std::lock_guard<std::mutex> s(stats_mu_);
                    stats_.requests_timeout++;
                }
                break;
            }
        }
        return batch;
    }

    // GenerationConfig -> one device request. Greedy (the fused argmax) when the reference's
    // rules reduce to the first maximum of the raw logits: temperature <= 0 without a repetition
    // penalty or a min_length mask (top-k and top-p keep the maximum); otherwise the slot samples
    // by TextGenerator::generate's rules.
    Request to_request(const Pending& p) const {
        const GenerationConfig& g = p.gen;
        if (g.num_beams > 1)
            throw std::invalid_argument("beam search (num_beams > 1) is not served by the device engine");
        if (!p.prompt.empty())
            throw std::invalid_argument(
                "decoder seed text is not supported: the device engine starts every request at "
                "BOS; pass the request text as its encoder input");
        Request r;
        r.source = p.source;
        r.max_length = g.max_length;
        r.bos = g.bos_token_id;
        r.stop_ids = {g.eos_token_id, g.pad_token_id};
        const bool greedy = g.temperature <= 0.0f && g.repetition_penalty == 1.0f && g.min_length <= 0;
        if (!greedy) {
            adai_b200_sampling s{};
            s.temperature = g.temperature;
            s.top_k = g.top_k;
            s.top_p = g.top_p;
            s.repetition_penalty = g.repetition_penalty;
            s.min_length = g.min_length;
            s.eos_token_id = g.eos_token_id;
            s.pad_token_id = g.pad_token_id;
            s.seed = seed_ ? static_cast<unsigned>(seed_ + p.number) : 0u;
            r.sampling = s;
        }
        return r;
    }

    void process(std::vector<Pending>& batch) {
        {
            std::lock_guard<std::mutex> s(stats_mu_);
            stats_.total_batches++;
            stats_.total_requests += batch.size();
        }
        std::vector<Request> reqs;
        std::vector<size_t> who;
        for (size_t i = 0; i < batch.size(); ++i) {
            try {
                reqs.push_back(to_request(batch[i]));
                who.push_back(i);
            } catch (...) {
                batch[i].result.set_exception(std::current_exception());
            }
        }
        std::vector<Result> res;
        try {
            BatchGenerator gen(kv_);
            res = gen.generate(reqs);
        } catch (...) {  // a device failure fails the whole batch it hit
            for (size_t i : who) batch[i].result.set_exception(std::current_exception());
            return;
        }
        for (size_t j = 0; j < who.size(); ++j) {
            Pending& p = batch[who[j]];
            if (!res[j].error.empty()) {
                p.result.set_exception(std::make_exception_ptr(std::runtime_error(res[j].error)));
                continue;
            }
            std::string text;
            try {
                text = tokenizer_->decode(res[j].tokens, true);
            } catch (...) {
                p.result.set_exception(std::current_exception());
                continue;
            }
            {
                std::lock_guard<std::mutex> s(stats_mu_);
                stats_.total_tokens_processed += res[j].tokens.empty() ? 0 : res[j].tokens.size() - 1;
            }
            p.result.set_value(std::move(text));
        }
    }

    KVArena& kv_;
    std::shared_ptr<Tokenizer> tokenizer_;
    EngineConfig config_;
    GenerationConfig default_gen_config_;
    uint32_t seed_;
    mutable std::mutex mu_;
    std::condition_variable cv_;
    std::queue<Pending> queue_;
    uint64_t submitted_ = 0;
    std::thread worker_;
    std::atomic<bool> running_;
    mutable std::mutex stats_mu_;
    EngineStats stats_;
};

}  // namespace adai_b200

#endif  // ADAI_B200_ENGINE_HPP
