// Host-only exercise of include/soc_b200_generation_context.hpp (no GPU): the tokenizer and
// generation-option wrappers, and GenerationContext's argument checks that fail before any
// device call.  Prints one "key: value" line per result for tests/test_cpp_mirror.py.
#include <cstdio>
#include <iostream>
#include <string>
#include <vector>

#include "soc_b200_generation_context.hpp"

static std::string ids_str(const std::vector<int>& v) {
    std::string s = "[";
    for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(v[i]);
    return s + "]";
}

int main(int argc, char** argv) {
    if (argc != 3) {
        std::cerr << "usage: mirror_check <manifest.json> <text>\n";
        return 2;
    }
    const std::string manifest = argv[1], text = argv[2];
    auto tok = soc::b200::Tokenizer::LoadFromManifest(manifest);
    const std::vector<int> ids = tok.Encode(text);
    std::cout << "ids: " << ids_str(ids) << "\n";
    std::cout << "roundtrip: " << (tok.Decode(ids) == text ? "ok" : "mismatch") << "\n";
    const std::string prompt = tok.BuildPrompt({{"user", text}}, true, false, "Be brief.");
    std::cout << "prompt_ids: " << ids_str(tok.Encode(prompt)) << "\n";
    const soc_generation_options g = soc::b200::GenerationOptionsFromManifest(manifest);
    std::cout << "options: " << g.max_new_tokens << " " << g.temperature << " " << g.top_k << " " << g.eos_token_id
              << " " << g.max_sequence_length << "\n";
    try {
        tok.Decode({1 << 30});
        std::cout << "decode_error: none\n";
    } catch (const std::exception& e) {
        std::cout << "decode_error: " << e.what() << "\n";
    }
    soc::b200::GenerationContext gen(nullptr, nullptr, 0, 8);
    std::string err;
    std::vector<float> logits;
    std::cout << "prefill_empty: " << gen.Prefill({}, &logits, &err) << " " << err << "\n";
    soc::b200::GenerationStepResult r;
    std::cout << "decode_unprefilled: " << gen.DecodeNextToken(5, &r, &err) << " " << err << "\n";
    std::vector<int> out;
    std::cout << "generate_too_long: " << gen.Generate(std::vector<int>(6, 1), 4, -1, &out, &err) << " " << err << "\n";
    std::cout << "generate_null: " << gen.Generate({1}, 1, -1, nullptr, &err) << " " << err << "\n";
    return 0;
}
