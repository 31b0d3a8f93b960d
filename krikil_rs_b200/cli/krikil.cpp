// krikil -- the command-line front end of src/main.rs on the GPU library:
// chat template -> tokenizer -> model (safetensors) -> device generation loop
// -> streamed text.  Same options, defaults, messages and exit codes as the
// reference's clap/anyhow CLI (src/main.rs:10-140), plus --device.
//
//   krikil [OPTIONS] <PROMPT>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <optional>
#include <string>
#include <vector>

#include "krikil.hpp"

namespace {

const char* const USAGE = "Usage: krikil [OPTIONS] <PROMPT>";

const char* const HELP =
    "Pebble-25M-Chat generation on a B200 GPU (the krikil command line)\n\n"
    "Usage: krikil [OPTIONS] <PROMPT>\n\n"
    "Arguments:\n"
    "  <PROMPT>  User prompt to generate a response for\n\n"
    "Options:\n"
    "  -m, --model <MODEL>                            Path to model safetensors weights [default: "
    "model.safetensors]\n"
    "      --tokenizer <TOKENIZER>                    Path to tokenizer.json file (defaults to sibling of model or "
    "./tokenizer.json)\n"
    "      --template <TEMPLATE>                      Path to Jinja chat template file (optional, defaults to "
    "built-in template)\n"
    "      --context <CONTEXT>                        Maximum context window length [default: 2048]\n"
    "      --max-tokens <MAX_TOKENS>                  Maximum new tokens to generate [default: 128]\n"
    "      --temp <TEMPERATURE>                       Sampling temperature (0.0 for greedy decoding) [default: 0.7]\n"
    "      --top-p <TOP_P>                            Nucleus sampling probability threshold [default: 0.95]\n"
    "      --top-k <TOP_K>                            Top-K filtering count [default: 50]\n"
    "      --repetition-penalty <REPETITION_PENALTY>  Repetition penalty factor [default: 1.2]\n"
    "      --seed <SEED>                              Random seed for deterministic generation\n"
    "      --quiet                                    Suppress timing and statistics printout at the end\n"
    "      --device <DEVICE>                          CUDA device ordinal [default: 0]\n"
    "  -h, --help                                     Print help\n"
    "  -V, --version                                  Print version\n";

struct Args {
    std::string model = "model.safetensors";
    std::optional<std::string> tokenizer, templ;
    size_t context = 2048, max_tokens = 128, top_k = 50;
    float temperature = 0.7f, top_p = 0.95f, repetition_penalty = 1.2f;
    std::optional<uint64_t> seed;
    bool quiet = false;
    int device = 0;
    std::optional<std::string> prompt;
};

[[noreturn]] void usage_error(const std::string& msg) {
    std::fprintf(stderr, "error: %s\n\n%s\n\nFor more information, try '--help'.\n", msg.c_str(), USAGE);
    std::exit(2);
}

template <typename T>
T parse_number(const std::string& flag, const std::string& v) {
    errno = 0;
    char* end = nullptr;
    T out{};
    if constexpr (std::is_floating_point<T>::value) {
        out = (T)std::strtod(v.c_str(), &end);
    } else if constexpr (std::is_signed<T>::value) {
        out = (T)std::strtoll(v.c_str(), &end, 10);
    } else {
        if (!v.empty() && v[0] == '-') end = nullptr;
        else out = (T)std::strtoull(v.c_str(), &end, 10);
    }
    if (v.empty() || !end || *end != '\0' || errno == ERANGE)
        usage_error("invalid value '" + v + "' for '" + flag + "'");
    return out;
}

Args parse(int argc, char** argv) {
    Args a;
    std::vector<std::string> av(argv + 1, argv + argc);
    bool positional_only = false;
    for (size_t i = 0; i < av.size(); ++i) {
        std::string arg = av[i];
        if (positional_only || arg.empty() || arg[0] != '-' || arg == "-") {
            if (a.prompt) usage_error("unexpected argument '" + arg + "' found");
            a.prompt = arg;
            continue;
        }
        if (arg == "--") {
            positional_only = true;
            continue;
        }
        if (arg == "-h" || arg == "--help") {
            std::fputs(HELP, stdout);
            std::exit(0);
        }
        if (arg == "-V" || arg == "--version") {
            std::puts("krikil 0.1.0");
            std::exit(0);
        }
        if (arg == "--quiet") {
            a.quiet = true;
            continue;
        }
        std::string flag = arg, value;
        bool have_value = false;
        const size_t eq = arg.find('=');
        if (arg.rfind("--", 0) == 0 && eq != std::string::npos) {
            flag = arg.substr(0, eq);
            value = arg.substr(eq + 1);
            have_value = true;
        } else if (arg.size() > 2 && arg[0] == '-' && arg[1] == 'm') {
            flag = "-m";
            value = arg.substr(2);
            have_value = true;
        }
        static const char* known[] = {"-m", "--model", "--tokenizer", "--template", "--context", "--max-tokens",
                                      "--temp", "--top-p", "--top-k", "--repetition-penalty", "--seed", "--device"};
        bool ok = false;
        for (const char* k : known) ok = ok || flag == k;
        if (!ok) usage_error("unexpected argument '" + arg + "' found");
        if (!have_value) {
            if (i + 1 >= av.size()) usage_error("a value is required for '" + flag + "' but none was supplied");
            value = av[++i];
        }
        if (flag == "-m" || flag == "--model") a.model = value;
        else if (flag == "--tokenizer") a.tokenizer = value;
        else if (flag == "--template") a.templ = value;
        else if (flag == "--context") a.context = parse_number<size_t>(flag, value);
        else if (flag == "--max-tokens") a.max_tokens = parse_number<size_t>(flag, value);
        else if (flag == "--temp") a.temperature = parse_number<float>(flag, value);
        else if (flag == "--top-p") a.top_p = parse_number<float>(flag, value);
        else if (flag == "--top-k") a.top_k = parse_number<size_t>(flag, value);
        else if (flag == "--repetition-penalty") a.repetition_penalty = parse_number<float>(flag, value);
        else if (flag == "--seed") a.seed = parse_number<uint64_t>(flag, value);
        else if (flag == "--device") a.device = parse_number<int>(flag, value);
    }
    if (!a.prompt) usage_error("the following required arguments were not provided:\n  <PROMPT>");
    return a;
}

// anyhow's report of an error with context: the context, then its cause.
[[noreturn]] void fail(const std::string& context, const std::string& cause) {
    if (cause.empty()) std::fprintf(stderr, "Error: %s\n", context.c_str());
    else std::fprintf(stderr, "Error: %s\n\nCaused by:\n    %s\n", context.c_str(), cause.c_str());
    std::exit(1);
}

// Rust's Debug text of a Duration: the largest unit that keeps an integer
// part, trailing zeros of the fraction dropped.
std::string fmt_duration(std::chrono::duration<double> d) {
    const uint64_t ns = (uint64_t)(d.count() * 1e9 + 0.5);
    auto frac = [](uint64_t v, int digits) {
        std::string s = std::to_string(v);
        s = std::string(digits - s.size(), '0') + s;
        while (!s.empty() && s.back() == '0') s.pop_back();
        return s.empty() ? std::string() : "." + s;
    };
    if (ns >= 1000000000ull) return std::to_string(ns / 1000000000ull) + frac(ns % 1000000000ull, 9) + "s";
    if (ns >= 1000000ull) return std::to_string(ns / 1000000ull) + frac(ns % 1000000ull, 6) + "ms";
    if (ns >= 1000ull) return std::to_string(ns / 1000ull) + frac(ns % 1000ull, 3) + "\xC2\xB5s";
    return std::to_string(ns) + "ns";
}

}  // namespace

int main(int argc, char** argv) {
    const Args args = parse(argc, argv);
    using krikil::Error;

    // 1. template engine
    std::optional<krikil::ChatTemplateEngine> templ;
    try {
        templ = args.templ ? krikil::ChatTemplateEngine::from_file(*args.templ)
                           : krikil::ChatTemplateEngine::default_template();
    } catch (const Error& e) {
        fail(e.what(), "");
    }
    // 2. tokenizer
    std::string tok_path;
    try {
        tok_path = krikil::PebbleTokenizer::resolve_path(args.model, args.tokenizer);
    } catch (const Error& e) {
        fail(e.what(), "");
    }
    std::optional<krikil::PebbleTokenizer> tokenizer;
    try {
        tokenizer.emplace(krikil::PebbleTokenizer::from_file(tok_path));
    } catch (const Error& e) {
        fail("Failed to load tokenizer from " + tok_path, e.what());
    }
    // 3. model
    std::optional<krikil::PebbleModel> model;
    try {
        model.emplace(krikil::PebbleModel::load_safetensors(args.model, args.device));
    } catch (const Error& e) {
        fail("Failed to load model from " + args.model, e.what());
    }
    // 4. prompt
    std::string formatted;
    try {
        formatted = templ->render_user_prompt(*args.prompt);
    } catch (const Error& e) {
        fail("Failed to format prompt with chat template", e.what());
    }
    std::vector<uint32_t> prompt_tokens;
    try {
        prompt_tokens = tokenizer->encode(formatted);
    } catch (const Error& e) {
        fail("Failed to tokenize formatted prompt", e.what());
    }
    if (prompt_tokens.empty()) fail("Prompt token sequence is empty", "");
    if (prompt_tokens.size() >= args.context)
        fail("Prompt length (" + std::to_string(prompt_tokens.size()) + " tokens) exceeds context limit (" +
                 std::to_string(args.context) + ")",
             "");
    try {
        // 5. state, 6. options, 7. generation (streams the text)
        krikil::PebbleState state(*model, args.context);
        krikil::GenerationOptions options;
        options.max_new_tokens = args.max_tokens;
        options.sampler_config.temperature = args.temperature;
        options.sampler_config.top_p = args.top_p;
        options.sampler_config.top_k = args.top_k;
        options.sampler_config.repetition_penalty = args.repetition_penalty;
        options.sampler_config.eos_token_id = tokenizer->eos_token_id();
        options.sampler_config.seed = args.seed;
        options.stream_stdout = true;
        krikil::GenerationEngine engine(*model, *tokenizer);
        const krikil::GenerationResult r = engine.generate(prompt_tokens, state, options);
        std::printf("\n");
        std::fflush(stdout);
        if (!args.quiet)
            std::fprintf(stderr,
                         "\n[Prompt: %zu tokens, Generated: %zu tokens | Prefill: %s, Decode: %s, Speed: %.2f "
                         "tok/s]\n",
                         r.prompt_token_count, r.generated_token_count, fmt_duration(r.prefill_duration).c_str(),
                         fmt_duration(r.decode_duration).c_str(), r.tokens_per_second);
    } catch (const Error& e) {
        fail(e.what(), "");
    }
    return 0;
}
