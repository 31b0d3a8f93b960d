/* krikil.hpp -- C++17 mirror of krikil-rs's public Rust API over the C ABI of
 * krikil_cuda.h (header only; link libkrikil_cuda).
 *
 * Same names, argument meanings and errors as the reference:
 *   PebbleModel::load_safetensors       src/model.rs:233-313
 *   PebbleModel::forward_prefill / step src/model.rs:316-368, 586-624
 *   PebbleState::new / reset            src/model.rs:204-229
 *   SamplerConfig, GenerationOptions,
 *   GenerationResult, GenerationEngine  src/sampler.rs:5-26, src/generate.rs:8-133
 * anyhow::Result errors become krikil::Error (what() = the reference's message,
 * status() = the krk_status code).  A PebbleState is one sequence (batch 1) as
 * in the reference; the batched C entry points remain available underneath. */
#pragma once

#include <chrono>
#include <cstdint>
#include <functional>
#include <optional>
#include <random>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "krikil_cuda.h"

namespace krikil {

class Error : public std::runtime_error {
   public:
    Error(int status, const std::string& msg) : std::runtime_error(msg), status_(status) {}
    int status() const { return status_; }

   private:
    int status_;
};

inline void check(int rc) {
    if (rc != KRK_OK) throw Error(rc, krk_last_error());
}

class PebbleState;

class PebbleModel {
   public:
    // src/model.rs:233
    static PebbleModel load_safetensors(const std::string& path, int device = 0) {
        krk_model* h = nullptr;
        check(krk_model_load(path.c_str(), device, &h));
        return PebbleModel(h);
    }
    PebbleModel(PebbleModel&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    PebbleModel& operator=(PebbleModel&& o) noexcept {
        if (this != &o) {
            reset_handle();
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    PebbleModel(const PebbleModel&) = delete;
    PebbleModel& operator=(const PebbleModel&) = delete;
    ~PebbleModel() { reset_handle(); }

    // src/model.rs:316: last-token logits [KRK_VOCAB]; advances current_pos by T
    std::vector<float> forward_prefill(const std::vector<uint32_t>& tokens, PebbleState& state) const;
    // src/model.rs:586
    std::vector<float> forward_step(uint32_t token, PebbleState& state) const;

    krk_model* handle() const { return h_; }

   private:
    explicit PebbleModel(krk_model* h) : h_(h) {}
    void reset_handle() {
        if (h_) krk_model_free(h_);
        h_ = nullptr;
    }
    krk_model* h_ = nullptr;
};

class PebbleState {
   public:
    // src/model.rs:204 PebbleState::new(&config, max_ctx)
    PebbleState(const PebbleModel& model, size_t max_ctx) : context_limit(max_ctx) {
        check(krk_state_create(model.handle(), 1, (int)max_ctx, &h_));
    }
    PebbleState(PebbleState&& o) noexcept : context_limit(o.context_limit), h_(std::exchange(o.h_, nullptr)) {}
    PebbleState(const PebbleState&) = delete;
    PebbleState& operator=(const PebbleState&) = delete;
    ~PebbleState() {
        if (h_) krk_state_free(h_);
    }
    // src/model.rs:221
    void reset() { check(krk_state_reset(h_, nullptr)); }
    size_t current_pos() const {
        int64_t p = 0;
        check(krk_state_positions(h_, &p));
        return (size_t)p;
    }
    krk_state* handle() const { return h_; }

    const size_t context_limit;

   private:
    krk_state* h_ = nullptr;
};

inline std::vector<float> PebbleModel::forward_prefill(const std::vector<uint32_t>& tokens,
                                                       PebbleState& state) const {
    std::vector<float> logits(KRK_VOCAB);
    const int32_t len = (int32_t)tokens.size();
    check(krk_prefill(h_, state.handle(), tokens.empty() ? nullptr : tokens.data(), &len, logits.data()));
    return logits;
}

inline std::vector<float> PebbleModel::forward_step(uint32_t token, PebbleState& state) const {
    std::vector<float> logits(KRK_VOCAB);
    check(krk_step(h_, state.handle(), &token, logits.data()));
    return logits;
}

// src/sampler.rs:5-26
struct SamplerConfig {
    float temperature = 0.7f;
    float top_p = 0.95f;
    size_t top_k = 50;
    float repetition_penalty = 1.2f;
    uint32_t eos_token_id = KRK_EOS_TOKEN;
    std::optional<uint64_t> seed;
};

// src/generate.rs:8-23
struct GenerationOptions {
    size_t max_new_tokens = 128;
    SamplerConfig sampler_config;
};

// src/generate.rs:25-34 (token ids; the tokenizer is not part of this library)
struct GenerationResult {
    std::vector<uint32_t> generated_tokens;
    std::chrono::duration<double> decode_duration{};
    size_t prompt_token_count = 0;
    size_t generated_token_count = 0;
    double tokens_per_second = 0.0;
};

// src/generate.rs:36-133: the whole loop, sampler included, on the device.
class GenerationEngine {
   public:
    explicit GenerationEngine(const PebbleModel& model) : model_(model) {}

    GenerationResult generate(const std::vector<uint32_t>& prompt_tokens, PebbleState& state,
                              const GenerationOptions& options,
                              const std::function<void(uint32_t)>& on_token = {}) const {
        const SamplerConfig& sc = options.sampler_config;
        if (sc.eos_token_id != KRK_EOS_TOKEN)
            throw Error(KRK_INVALID, "the device generation loop stops at token " + std::to_string(KRK_EOS_TOKEN));
        GenerationResult r;
        r.prompt_token_count = prompt_tokens.size();
        if (options.max_new_tokens == 0) return r;
        std::vector<uint32_t> toks(options.max_new_tokens);
        int32_t n = 0;
        const int32_t len = (int32_t)prompt_tokens.size();
        const auto t0 = std::chrono::steady_clock::now();
        if (sc.temperature <= 1e-6f) {
            check(krk_generate_greedy(model_.handle(), state.handle(), prompt_tokens.data(), &len,
                                      (int)options.max_new_tokens, sc.repetition_penalty, 1, toks.data(), &n));
        } else {
            // SamplerConfig::seed None: StdRng::from_entropy
            const uint64_t seed = sc.seed ? *sc.seed : ((uint64_t)std::random_device{}() << 32) ^ std::random_device{}();
            check(krk_generate_sample(model_.handle(), state.handle(), prompt_tokens.data(), &len,
                                      (int)options.max_new_tokens, sc.temperature, sc.top_p, (int)sc.top_k,
                                      sc.repetition_penalty, &seed, 1, toks.data(), &n));
        }
        r.decode_duration = std::chrono::steady_clock::now() - t0;
        toks.resize((size_t)n);
        if (on_token)
            for (uint32_t t : toks) on_token(t);
        r.generated_tokens = std::move(toks);
        r.generated_token_count = r.generated_tokens.size();
        const double secs = r.decode_duration.count();
        r.tokens_per_second = secs > 0 ? r.generated_token_count / secs : 0.0;
        return r;
    }

   private:
    const PebbleModel& model_;
};

}  // namespace krikil
