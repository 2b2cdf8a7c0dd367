// soc_b200_cli: the reference's command-line runner (Mac/cpu/main.cpp) over the C ABI.
//
// Same flags, defaults, output lines and error behaviour: options come from the manifest's
// generation_config and are overridden by the flags given (main.cpp:87-106); the prompt is
// optionally wrapped by the Qwen3 chat template (RuntimePipeline::PreparePrompt,
// runtime_pipeline.cpp:57-71); generation is greedy with an optional EOS stop into a KV cache
// of max_sequence_length positions (GenerationSession::Generate, generation_session.cpp:46-83).
// Any failure prints "runtime error: <message>" and the usage text and exits 1.
//
// One extra option, --weight-format native|f16|bf16|int8|int4, picks the stored format of
// the block linears on the device (default: the bundle's own).

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "soc_b200.h"

namespace {

struct Options {
    std::string manifest, prompt, system_prompt;
    soc_generation_options gen{};
    bool set_max_new = false, set_temperature = false, set_top_k = false, set_eos = false, set_max_seq = false;
    bool chat = false, thinking = true;
    int weight_format = SOC_B200_WEIGHTS_NATIVE;
    int device = 0;
};

[[noreturn]] void usage(const char* exe, int code) {
    std::cerr << "Usage: " << exe << " --manifest <manifest.json> --prompt <text> [options]\n"
              << "Options:\n"
              << "  --max-new-tokens <n>   Number of tokens to generate (default: 32)\n"
              << "  --temperature <value>  Sampler temperature (default: 1.0)\n"
              << "  --top-k <n>            Sampler top-k (default: 1)\n"
              << "  --eos-token-id <id>    Stop when this token id is generated (default: disabled)\n"
              << "  --max-seq-len <n>      KV cache capacity for generation (default: 256)\n"
              << "  --apply-chat-template  Wrap prompt as a single user chat turn using tokenizer runtime template\n"
              << "  --disable-thinking     Omit the opening <think> tag when applying the chat template\n"
              << "  --system-prompt <txt>  Override the default system prompt used by the chat template\n"
              << "  --weight-format <f>    Device format of the block linears: native, f16, bf16, int8, int4\n"
              << "  --device <n>           CUDA device (default: 0)\n";
    std::exit(code);
}

void check(int rc) {
    if (rc != SOC_B200_OK) throw std::runtime_error(soc_b200_last_error());
}

Options parse(int argc, char** argv) {
    Options o;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto value = [&](const char* name) -> std::string {
            if (i + 1 >= argc) throw std::runtime_error(std::string("missing value for argument: ") + name);
            return argv[++i];
        };
        if (a == "--manifest") {
            o.manifest = value("--manifest");
        } else if (a == "--prompt") {
            o.prompt = value("--prompt");
        } else if (a == "--max-new-tokens") {
            o.gen.max_new_tokens = static_cast<size_t>(std::stoull(value("--max-new-tokens")));
            o.set_max_new = true;
        } else if (a == "--temperature") {
            o.gen.temperature = std::stof(value("--temperature"));
            o.set_temperature = true;
        } else if (a == "--top-k") {
            o.gen.top_k = static_cast<size_t>(std::stoull(value("--top-k")));
            o.set_top_k = true;
        } else if (a == "--eos-token-id") {
            o.gen.eos_token_id = std::stoi(value("--eos-token-id"));
            o.set_eos = true;
        } else if (a == "--max-seq-len") {
            o.gen.max_sequence_length = static_cast<size_t>(std::stoull(value("--max-seq-len")));
            o.set_max_seq = true;
        } else if (a == "--apply-chat-template") {
            o.chat = true;
        } else if (a == "--disable-thinking") {
            o.thinking = false;
        } else if (a == "--system-prompt") {
            o.system_prompt = value("--system-prompt");
        } else if (a == "--weight-format") {
            const std::string f = value("--weight-format");
            if (f == "native") o.weight_format = SOC_B200_WEIGHTS_NATIVE;
            else if (f == "f16") o.weight_format = SOC_B200_WEIGHTS_F16;
            else if (f == "bf16") o.weight_format = SOC_B200_WEIGHTS_BF16;
            else if (f == "int8") o.weight_format = SOC_B200_WEIGHTS_INT8_G64;
            else if (f == "int4") o.weight_format = SOC_B200_WEIGHTS_INT4_G32;
            else throw std::runtime_error("unknown weight format: " + f);
        } else if (a == "--device") {
            o.device = std::stoi(value("--device"));
        } else if (a == "--help" || a == "-h") {
            usage(argv[0], 0);
        } else {
            throw std::runtime_error("unknown argument: " + a);
        }
    }
    if (o.manifest.empty()) throw std::runtime_error("--manifest is required");
    if (o.prompt.empty()) throw std::runtime_error("--prompt is required");
    return o;
}

void print_ids(const char* label, const std::vector<int32_t>& ids) {
    std::cout << label << ": [";
    for (size_t i = 0; i < ids.size(); ++i) std::cout << (i ? ", " : "") << ids[i];
    std::cout << "]\n";
}

// RAII holders so an error path releases the device objects before the process exits.
struct Handles {
    soc_ctx* ctx = nullptr;
    soc_model* model = nullptr;
    soc_kv* kv = nullptr;
    soc_tokenizer* tok = nullptr;
    ~Handles() {
        if (kv) soc_b200_free_kv(kv);
        if (model) soc_b200_free_model(model);
        if (ctx) soc_b200_close(ctx);
        if (tok) soc_b200_tokenizer_free(tok);
    }
};

std::string tokenizer_path(const std::string& manifest) {
    size_t n = 0;
    soc_b200_manifest_tokenizer_path(manifest.c_str(), nullptr, 0, &n);
    std::vector<char> buf(n + 1);
    check(soc_b200_manifest_tokenizer_path(manifest.c_str(), buf.data(), buf.size(), &n));
    return std::string(buf.data(), n);
}

std::string chat_prompt(const soc_tokenizer* tok, const Options& o) {
    const char* roles[1] = {"user"};
    const char* contents[1] = {o.prompt.c_str()};
    size_t n = 0;
    std::string out(o.prompt.size() + o.system_prompt.size() + 1024, '\0');
    int rc = soc_b200_chat_prompt(tok, roles, contents, 1, 1, o.thinking, o.system_prompt.c_str(), &out[0],
                                  out.size(), &n);
    if (rc == SOC_B200_ERR_CAPACITY) {
        out.assign(n, '\0');
        rc = soc_b200_chat_prompt(tok, roles, contents, 1, 1, o.thinking, o.system_prompt.c_str(), &out[0],
                                  out.size(), &n);
    }
    check(rc);
    out.resize(n);
    return out;
}

int run(const Options& cli) {
    Handles h;
    // RuntimePipeline::LoadBundle: manifest, tokenizer, their cross checks and the tensor
    // records, all on the host (a broken bundle is reported before the GPU is touched), then
    // the model.
    check(soc_b200_validate_bundle(cli.manifest.c_str()));
    check(soc_b200_tokenizer_load(tokenizer_path(cli.manifest).c_str(), &h.tok));
    check(soc_b200_open(cli.device, &h.ctx));
    check(soc_b200_load_bundle(h.ctx, cli.manifest.c_str(), cli.weight_format, 0, 1, nullptr, &h.model));
    soc_model_info info{};
    check(soc_b200_model_info(h.model, &info));
    check(soc_b200_tokenizer_check_model(h.tok, info.vocab));

    soc_generation_options g{};
    check(soc_b200_manifest_generation_options(cli.manifest.c_str(), &g));
    if (cli.set_max_new) g.max_new_tokens = cli.gen.max_new_tokens;
    if (cli.set_temperature) g.temperature = cli.gen.temperature;
    if (cli.set_top_k) g.top_k = cli.gen.top_k;
    if (cli.set_eos) g.eos_token_id = cli.gen.eos_token_id;
    if (cli.set_max_seq) g.max_sequence_length = cli.gen.max_sequence_length;
    check(soc_b200_set_sampler(h.model, g.temperature, g.top_k));
    if (g.max_sequence_length == 0) throw std::runtime_error("kv cache requires positive max_sequence_length");

    const std::string prepared = cli.chat ? chat_prompt(h.tok, cli) : cli.prompt;
    std::vector<int32_t> prompt_ids(prepared.size() + 16);
    int n_prompt = 0;
    check(soc_b200_tokenizer_encode(h.tok, prepared.data(), prepared.size(), prompt_ids.data(),
                                    static_cast<int>(prompt_ids.size()), &n_prompt));
    prompt_ids.resize(n_prompt);

    std::vector<int32_t> generated;
    const size_t cap = g.max_sequence_length;
    if (g.max_new_tokens != 0) {
        // The reference caches the prompt and every generated token but the last; a write past
        // the cache's max_sequence_length positions fails at the step that would make it.
        if (prompt_ids.size() > cap) throw std::runtime_error("kv cache write position out of range");
        const size_t room = cap - prompt_ids.size() + 1;
        const size_t steps = std::min(g.max_new_tokens, room);
        check(soc_b200_kv_create(h.model, 1, static_cast<int>(cap), 16, &h.kv));
        generated.resize(steps);
        int n_out = 0;
        check(soc_b200_generate(h.model, h.kv, 0, prompt_ids.data(), n_prompt, static_cast<int>(steps),
                                g.eos_token_id, generated.data(), &n_out));
        generated.resize(n_out);
        const bool stopped = g.eos_token_id >= 0 && n_out > 0 && generated.back() == g.eos_token_id;
        if (!stopped && static_cast<size_t>(n_out) < g.max_new_tokens)
            throw std::runtime_error("kv cache write position out of range");
    }

    std::string text(64 + 64 * generated.size(), '\0');
    size_t n_text = 0;
    int rc = soc_b200_tokenizer_decode(h.tok, generated.data(), static_cast<int>(generated.size()), &text[0],
                                       text.size(), &n_text);
    if (rc == SOC_B200_ERR_CAPACITY) {
        text.assign(n_text, '\0');
        rc = soc_b200_tokenizer_decode(h.tok, generated.data(), static_cast<int>(generated.size()), &text[0],
                                       text.size(), &n_text);
    }
    check(rc);
    text.resize(n_text);

    std::cout << "prompt: " << cli.prompt << "\n";
    if (prepared != cli.prompt) std::cout << "serialized_prompt: " << prepared << "\n";
    print_ids("prompt_token_ids", prompt_ids);
    print_ids("generated_token_ids", generated);
    std::cout << "generated_text: " << text << "\n";
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        return run(parse(argc, argv));
    } catch (const std::exception& e) {
        std::cerr << "runtime error: " << e.what() << "\n";
        usage(argv[0], 1);
    }
}
