// ref_runner.cpp -- command-line driver of the PokitLMs reference decoder
// (test infrastructure only; the product library never links it).
//
// Loads a Qwen3-MoE GGUF with the reference's own Qwen3MoeRunner (compiled
// from its unmodified sources by `make -C oracle runner`) and greedy-decodes
// from a prompt of token ids, exactly as its generate_tokens does
// (src/qwen3_moe_runner.cpp:751-821: prefill with logits for the last prompt
// token, greedy argmax sampling, stop at EOS).  The expert cache budget is
// set high enough that no expert is read twice from disk.  With --qwen35 the
// model is a Qwen3.5 GGUF run by Qwen35Runner (src/qwen35_runner.cpp:845-913,
// default KV window and FP16 KV cache).
//
//   ref_runner [--qwen35] MODEL.gguf PROMPT_IDS_FILE MAX_NEW [LOGITS_OUT]
//
// PROMPT_IDS_FILE holds whitespace-separated token ids.  Prints one JSON line
// {"ids": [...], "prefill_ns": N, "decode_ns": N, "generated": N}.  With
// LOGITS_OUT, first writes the float32 logits after the last prompt token
// (Qwen3MoeRunner::forward_token over the prompt) to that file.
#include "pokitlms/model/qwen35_runner.hpp"
#include "pokitlms/model/qwen3_moe_runner.hpp"

#include <cstdint>
#include <cstdio>
#include <exception>
#include <fstream>
#include <string>
#include <vector>

namespace {

template <typename Runner, typename Generate>
int run(Runner& runner, const std::vector<std::uint32_t>& prompt, int argc, char** argv, Generate generate) {
    if (argc > 4) {
        std::vector<float> logits;
        for (std::size_t i = 0; i < prompt.size(); ++i) logits = runner.forward_token(prompt[i], i);
        std::ofstream out(argv[4], std::ios::binary);
        out.write(reinterpret_cast<const char*>(logits.data()),
                  static_cast<std::streamsize>(logits.size() * sizeof(float)));
        runner.reset();
    }
    std::uint64_t prefill = 0, decode = 0;
    std::size_t generated = 0;
    const auto ids = generate(prefill, decode, generated);
    std::printf("{\"ids\": [");
    for (std::size_t i = 0; i < ids.size(); ++i) std::printf("%s%u", i ? ", " : "", ids[i]);
    std::printf("], \"prefill_ns\": %llu, \"decode_ns\": %llu, \"generated\": %zu}\n",
                static_cast<unsigned long long>(prefill), static_cast<unsigned long long>(decode), generated);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const bool qwen35 = argc > 1 && std::string(argv[1]) == "--qwen35";
    if (qwen35) {
        --argc;
        ++argv;
    }
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s [--qwen35] MODEL.gguf PROMPT_IDS_FILE MAX_NEW [LOGITS_OUT]\n", argv[0]);
        return 2;
    }
    try {
        std::vector<std::uint32_t> prompt;
        {
            std::ifstream in(argv[2]);
            std::uint64_t v = 0;
            while (in >> v) prompt.push_back(static_cast<std::uint32_t>(v));
        }
        const std::size_t max_new = std::stoul(argv[3]);
        if (qwen35) {
            pokitlms::model::Qwen35Runner runner(argv[1]);
            return run(runner, prompt, argc, argv, [&](std::uint64_t& p, std::uint64_t& d, std::size_t& g) {
                pokitlms::model::Qwen35GenerationStats stats{};
                auto ids = runner.generate_tokens(prompt, max_new, &stats);
                p = stats.prefill_time_ns;
                d = stats.decode_time_ns;
                g = stats.generated_tokens;
                return ids;
            });
        }
        const std::size_t budget = std::size_t(64) << 30;
        pokitlms::model::Qwen3MoeRunner runner(argv[1], budget);
        return run(runner, prompt, argc, argv, [&](std::uint64_t& p, std::uint64_t& d, std::size_t& g) {
            pokitlms::model::GenerationOptions options{};       // temperature 0: greedy
            pokitlms::model::GenerationStats stats{};
            auto ids = runner.generate_tokens(prompt, max_new, options, &stats);
            p = stats.prefill_time_ns;
            d = stats.decode_time_ns;
            g = stats.generated_tokens;
            return ids;
        });
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_runner: %s\n", e.what());
        return 1;
    }
}
