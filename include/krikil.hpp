/* krikil.hpp -- C++17 mirror of krikil-rs's public Rust API over the C ABI of
 * krikil_cuda.h (header only; link libkrikil_cuda).
 *
 * Same names, argument meanings and errors as the reference:
 *   PebbleModel::load_safetensors       src/model.rs:233-313
 *   PebbleModel::forward_prefill / step src/model.rs:316-368, 586-624
 *   PebbleState::new / reset            src/model.rs:204-229
 *   SamplerConfig, GenerationOptions,
 *   GenerationResult, GenerationEngine  src/sampler.rs:5-26, src/generate.rs:8-133
 *   PebbleTokenizer                     src/tokenizer.rs:7-80
 *   ChatMessage, ChatTemplateEngine     src/template.rs:9-79
 * anyhow::Result errors become krikil::Error (what() = the reference's message,
 * status() = the krk_status code).  A PebbleState is one sequence (batch 1) as
 * in the reference; the batched C entry points remain available underneath. */
#pragma once

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <functional>
#include <iostream>
#include <optional>
#include <random>
#include <stdexcept>
#include <string>
#include <utility>
#include <sstream>
#include <vector>

#include "krikil_cuda.h"
#include "krikil_text.h"

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

// ------------------------------------------------------------ text front end
// src/tokenizer.rs:5
constexpr uint32_t DEFAULT_EOS_TOKEN_ID = 0;

namespace detail {
// Runs call(buf, cap, &len) under the size-query rule of krikil_text.h.
template <typename F>
std::string read_string(F&& call) {
    size_t len = 0;
    std::string out(256, '\0');
    int rc = call(&out[0], out.size(), &len);
    if (rc == KRK_INVALID && len > out.size()) {
        out.assign(len, '\0');
        rc = call(&out[0], out.size(), &len);
    }
    check(rc);
    out.resize(len);
    return out;
}
}  // namespace detail

// src/tokenizer.rs:7-80 (a byte-level BPE read from tokenizer.json)
class PebbleTokenizer {
   public:
    static PebbleTokenizer from_file(const std::string& path) {
        krk_tokenizer* h = nullptr;
        check(krk_tokenizer_load(path.c_str(), &h));
        return PebbleTokenizer(h);
    }
    PebbleTokenizer(PebbleTokenizer&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    PebbleTokenizer(const PebbleTokenizer&) = delete;
    PebbleTokenizer& operator=(const PebbleTokenizer&) = delete;
    ~PebbleTokenizer() {
        if (h_) krk_tokenizer_free(h_);
    }

    std::vector<uint32_t> encode(const std::string& text) const {
        std::vector<uint32_t> ids(text.size() + 1);
        size_t n = 0;
        check(krk_tokenizer_encode(h_, text.data(), text.size(), ids.data(), ids.size(), &n));
        ids.resize(n);
        return ids;
    }
    // special tokens skipped
    std::string decode(const std::vector<uint32_t>& tokens) const { return decode_ids(tokens, true); }
    // one token, special tokens kept
    std::string decode_token(uint32_t token) const { return decode_ids({token}, false); }
    uint32_t eos_token_id() const {
        uint32_t id = 0;
        check(krk_tokenizer_eos_token_id(h_, &id));
        return id;
    }
    size_t vocab_size() const {
        size_t n = 0;
        check(krk_tokenizer_vocab_size(h_, &n));
        return n;
    }
    static std::string resolve_path(const std::string& model_path,
                                    const std::optional<std::string>& explicit_tokenizer = std::nullopt) {
        return detail::read_string([&](char* b, size_t cap, size_t* n) {
            return krk_tokenizer_resolve_path(model_path.c_str(),
                                              explicit_tokenizer ? explicit_tokenizer->c_str() : nullptr, b, cap, n);
        });
    }

   private:
    explicit PebbleTokenizer(krk_tokenizer* h) : h_(h) {}
    std::string decode_ids(const std::vector<uint32_t>& ids, bool skip_special) const {
        return detail::read_string([&](char* b, size_t cap, size_t* n) {
            return krk_tokenizer_decode(h_, ids.data(), ids.size(), skip_special ? 1 : 0, b, cap, n);
        });
    }
    krk_tokenizer* h_ = nullptr;
};

// src/template.rs:9-29
struct ChatMessage {
    std::string role;
    std::string content;
    static ChatMessage user(std::string c) { return {"user", std::move(c)}; }
    static ChatMessage assistant(std::string c) { return {"assistant", std::move(c)}; }
};

// src/template.rs:31-79
class ChatTemplateEngine {
   public:
    explicit ChatTemplateEngine(std::string template_source) : src_(std::move(template_source)) {}
    static ChatTemplateEngine from_file(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw Error(KRK_IO, "Failed to read chat template from " + path);
        std::ostringstream ss;
        ss << f.rdbuf();
        return ChatTemplateEngine(ss.str());
    }
    static ChatTemplateEngine default_template() { return ChatTemplateEngine(krk_default_chat_template()); }

    std::string render(const std::vector<ChatMessage>& messages, bool add_generation_prompt) const {
        std::vector<const char*> roles, contents;
        for (const auto& m : messages) {
            roles.push_back(m.role.c_str());
            contents.push_back(m.content.c_str());
        }
        return detail::read_string([&](char* b, size_t cap, size_t* n) {
            return krk_chat_template_render(src_.c_str(), roles.data(), contents.data(), messages.size(),
                                            add_generation_prompt ? 1 : 0, b, cap, n);
        });
    }
    std::string render_user_prompt(const std::string& prompt) const {
        return render({ChatMessage::user(prompt)}, true);
    }
    const std::string& template_source() const { return src_; }

   private:
    std::string src_;
};

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
    bool stream_stdout = true;  // print each token's text (needs the engine's tokenizer)
};

// src/generate.rs:25-34.  The device loop runs prefill and decode in one call:
// decode_duration covers both and prefill_duration stays zero.
struct GenerationResult {
    std::string generated_text;  // decode_token of each generated token, concatenated (needs a tokenizer)
    std::vector<uint32_t> generated_tokens;
    std::chrono::duration<double> prefill_duration{};
    std::chrono::duration<double> decode_duration{};
    size_t prompt_token_count = 0;
    size_t generated_token_count = 0;
    double tokens_per_second = 0.0;
};

// src/generate.rs:36-133: the whole loop, sampler included, on the device.
// Token text (stdout stream, callback, generated_text) follows once the loop
// has returned, in token order.
class GenerationEngine {
   public:
    GenerationEngine(const PebbleModel& model, const PebbleTokenizer& tokenizer)
        : model_(model), tokenizer_(&tokenizer) {}
    explicit GenerationEngine(const PebbleModel& model) : model_(model) {}  // token ids only

    // src/generate.rs:46-53
    GenerationResult generate(const std::vector<uint32_t>& prompt_tokens, PebbleState& state,
                              const GenerationOptions& options) const {
        return generate_with_callback(prompt_tokens, state, options, [](const std::string&) {});
    }

    // src/generate.rs:55-133: on_token receives each token's text
    GenerationResult generate_with_callback(const std::vector<uint32_t>& prompt_tokens, PebbleState& state,
                                            const GenerationOptions& options,
                                            const std::function<void(const std::string&)>& on_token) const {
        GenerationResult r = generate(prompt_tokens, state, options, std::function<void(uint32_t)>{});
        if (!tokenizer_) return r;
        for (uint32_t t : r.generated_tokens) {
            std::string text;
            try {
                text = tokenizer_->decode_token(t);
            } catch (const Error&) {  // src/generate.rs:89-92: a token that does not decode prints nothing
            }
            if (options.stream_stdout) {
                std::fwrite(text.data(), 1, text.size(), stdout);
                std::fflush(stdout);
            }
            if (on_token) on_token(text);
            r.generated_text += text;
        }
        return r;
    }

    // The same loop with a callback per token id.
    GenerationResult generate(const std::vector<uint32_t>& prompt_tokens, PebbleState& state,
                              const GenerationOptions& options, const std::function<void(uint32_t)>& on_token) const {
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
    const PebbleTokenizer* tokenizer_ = nullptr;
};

}  // namespace krikil
