// The reference's public API driven through include/krikil.hpp, in the shape
// of its own Rust tests (src/model.rs:791-932 forward_prefill / forward_step,
// src/generate.rs generation): run by tests/test_cpp_api.py, which compares
// the values written to the output file against the oracle.
//
// usage: test_api <weights.safetensors> <out.bin> <tokenizer.json>
// exit 0: all checks passed; 77: no CUDA device (only the loader checks ran);
// 1: a check failed (message on stderr).
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "krikil.hpp"

using krikil::Error;

static int failures = 0;
#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            std::fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            ++failures;                                                      \
        }                                                                    \
    } while (0)

template <typename F>
static void expect_error(F&& f, int status, const char* needle) {
    try {
        f();
        std::fprintf(stderr, "expected error %d (%s), got none\n", status, needle);
        ++failures;
    } catch (const Error& e) {
        if (e.status() != status || std::strstr(e.what(), needle) == nullptr) {
            std::fprintf(stderr, "expected error %d containing '%s', got %d '%s'\n", status, needle, e.status(),
                         e.what());
            ++failures;
        }
    }
}

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: test_api <weights> <out> <tokenizer.json>\n");
        return 2;
    }
    // text front end (src/tokenizer.rs, src/template.rs): host only
    {
        auto tok = krikil::PebbleTokenizer::from_file(argv[3]);
        const auto tmpl = krikil::ChatTemplateEngine::default_template();
        const std::string prompt = tmpl.render_user_prompt("What is the capital of France?");
        CHECK(prompt == "user: What is the capital of France? assistant: ");
        const auto ids = tok.encode(prompt);
        CHECK(!ids.empty() && tok.decode(ids) == prompt);
        CHECK(tok.eos_token_id() == krikil::DEFAULT_EOS_TOKEN_ID && tok.decode_token(0) == "<|eos|>");
        CHECK(tmpl.render({krikil::ChatMessage::user("Hello"), krikil::ChatMessage::assistant("Hi there!")}, false) ==
              "user: Hello assistant: Hi there! ");
        expect_error([] { krikil::ChatTemplateEngine("{% if %}").render({}, false); }, KRK_INVALID,
                     "Failed to parse Jinja chat template");
        expect_error([] { krikil::PebbleTokenizer::from_file("/nonexistent/tokenizer.json"); }, KRK_IO,
                     "Failed to load tokenizer from");
    }
    // load errors come before any device work (src/model.rs:233-240)
    expect_error([] { krikil::PebbleModel::load_safetensors("/nonexistent/model.safetensors"); }, KRK_IO,
                 "Failed to open model file");
    krk_model* probe = nullptr;
    if (krk_model_load(argv[1], 0, &probe) == KRK_CUDA) {
        std::printf("no CUDA device: loader checks only (%d failures)\n", failures);
        return failures ? 1 : 77;
    }
    krk_model_free(probe);

    FILE* out = std::fopen(argv[2], "wb");
    if (!out) return 2;
    auto model = krikil::PebbleModel::load_safetensors(argv[1]);
    krikil::PebbleState state(model, 64);
    std::vector<uint32_t> prompt;
    for (uint32_t i = 0; i < 12; ++i) prompt.push_back((i * 397u + 11u) % KRK_VOCAB);

    // forward_prefill then forward_step (src/model.rs:862-931)
    std::vector<float> lp = model.forward_prefill(prompt, state);
    CHECK(lp.size() == (size_t)KRK_VOCAB && state.current_pos() == prompt.size());
    std::vector<float> ls = model.forward_step(199, state);
    CHECK(state.current_pos() == prompt.size() + 1);
    std::fwrite(lp.data(), 4, lp.size(), out);
    std::fwrite(ls.data(), 4, ls.size(), out);

    // errors leave the state untouched (src/model.rs:317-335, 587-593)
    expect_error([&] { model.forward_step(4096, state); }, KRK_BAD_TOKEN, "exceeds vocab size");
    expect_error([&] { model.forward_prefill({}, state); }, KRK_EMPTY, "Cannot prefill empty sequence");
    CHECK(state.current_pos() == prompt.size() + 1);
    krikil::PebbleState small(model, 8);
    expect_error([&] { model.forward_prefill(std::vector<uint32_t>(9, 1u), small); }, KRK_CONTEXT_OVERFLOW,
                 "exceeds context limit");
    state.reset();
    CHECK(state.current_pos() == 0);

    // generation (src/generate.rs:55-133): greedy with penalty, then seeded sampling
    krikil::GenerationEngine engine(model);
    krikil::GenerationOptions opt;
    opt.max_new_tokens = 10;
    opt.sampler_config.temperature = 0.0f;
    opt.sampler_config.repetition_penalty = 1.2f;
    size_t streamed = 0;
    auto g = engine.generate(prompt, state, opt, [&](uint32_t) { ++streamed; });
    CHECK(streamed == g.generated_tokens.size() && g.prompt_token_count == prompt.size());
    const uint32_t ng = (uint32_t)g.generated_tokens.size();
    std::fwrite(&ng, 4, 1, out);
    std::fwrite(g.generated_tokens.data(), 4, ng, out);
    opt.sampler_config = krikil::SamplerConfig{};  // reference defaults: T 0.7, top-p 0.95, top-k 50, penalty 1.2
    opt.sampler_config.seed = 42;
    auto r1 = engine.generate(prompt, state, opt);
    auto r2 = engine.generate(prompt, state, opt);
    CHECK(r1.generated_tokens == r2.generated_tokens);  // src/sampler.rs:185-201, seeded determinism
    const uint32_t ns = (uint32_t)r1.generated_tokens.size();
    std::fwrite(&ns, 4, 1, out);
    std::fwrite(r1.generated_tokens.data(), 4, ns, out);
    std::fclose(out);
    std::printf("%d failures\n", failures);
    return failures ? 1 : 0;
}
