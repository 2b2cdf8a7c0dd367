// C++ host-side mirror of the reference runtime's GenerationContext over the
// soc_b200 C ABI (header-only).
//
// Same call shape as soc::gpu::GenerationContext (Mac/gpu/include/runtime/
// generation_context.h:23-74): bool-returning Prefill / DecodeNextToken /
// Generate with a nullable std::string* error_message, Reset(), and the prompt
// / running token id accessors.  The Metal-specific arguments (MetalContext,
// PipelineCache*, BufferArena*) have no B200 counterpart: device, stream and
// buffers live in the soc_ctx / soc_model / soc_kv handles.  The next-token pick
// happens on the device (the model's Sampler, soc_b200_set_sampler), so only the
// token id -- and the logits row when asked for -- crosses PCIe.
//
// Also here: Tokenizer (TokenizerRuntime + Qwen3TemplateBuilder, Mac/cpu/header/
// tokenizer_runtime.h:12-46, runtime_assets.cpp:221-258) and
// GenerationOptionsFromManifest (RuntimePipeline, runtime_pipeline.cpp:43-55), which
// throw std::runtime_error with the library's message as the reference does.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "soc_b200.h"

namespace soc::b200 {

struct GenerationStepResult {
    int token_id = -1;
    std::vector<float> top_logits;   // the sampler's top_k candidates, larger first (generation_context.h:17-21)
    std::vector<int> top_token_ids;
    std::vector<float> logits;       // the whole row, filled when requested
};

class GenerationContext {
public:
    // `model` and `kv` stay owned by the caller; `seq` is this context's slot in `kv`.
    // `top_k`: candidates per step in GenerationStepResult (the Sampler's top_k, 1..64).
    GenerationContext(soc_model* model, soc_kv* kv, int seq, std::size_t max_sequence_length, std::size_t top_k = 1)
        : model_(model), kv_(kv), seq_(seq), max_sequence_length_(max_sequence_length),
          top_k_(top_k < 1 ? 1 : (top_k > 64 ? 64 : top_k)) {
        soc_b200_model_info(model_, &info_);
    }

    // generation_context.cpp:17-59: reset, then run the prompt; logits of the last row
    // go to *last_logits when it is non-null.
    bool Prefill(const std::vector<int>& token_ids, std::vector<float>* last_logits, std::string* error_message) {
        if (token_ids.empty()) return Fail("GenerationContext prefill requires at least one token", error_message);
        if (token_ids.size() > max_sequence_length_)
            return Fail("GenerationContext sequence length would exceed max_sequence_length", error_message);
        Reset();
        std::vector<int32_t> ids(token_ids.begin(), token_ids.end());
        std::vector<float> row;
        if (last_logits) row.resize(static_cast<std::size_t>(info_.vocab));
        int32_t next = -1;
        if (soc_b200_prefill(model_, kv_, seq_, ids.data(), static_cast<int>(ids.size()),
                             last_logits ? row.data() : nullptr, &next) != SOC_B200_OK)
            return Fail(soc_b200_last_error(), error_message);
        if (last_logits) *last_logits = std::move(row);
        prompt_token_ids_ = token_ids;
        running_token_ids_ = token_ids;
        prefill_next_ = next;
        return true;
    }

    // generation_context.cpp:61-116: the tail and length checks, one step, greedy pick.
    bool DecodeNextToken(int last_token_id, GenerationStepResult* result, std::string* error_message,
                         bool want_logits = false) {
        if (result == nullptr) return Fail("GenerationContext decode requires a non-null result", error_message);
        if (running_token_ids_.empty())
            return Fail("GenerationContext decode requires a prefilled KV cache", error_message);
        if (running_token_ids_.back() != last_token_id)
            return Fail("GenerationContext decode requires last_token_id to match the current sequence tail",
                        error_message);
        if (running_token_ids_.size() >= max_sequence_length_)
            return Fail("GenerationContext sequence length would exceed max_sequence_length", error_message);
        const int seq = seq_;
        const int32_t last = last_token_id;
        int32_t next = -1;
        if (want_logits) result->logits.resize(static_cast<std::size_t>(info_.vocab));
        if (soc_b200_decode(model_, kv_, 1, &seq, &last, want_logits ? result->logits.data() : nullptr, &next) !=
            SOC_B200_OK)
            return Fail(soc_b200_last_error(), error_message);
        result->token_id = next;
        result->top_logits.resize(top_k_);
        std::vector<int32_t> ids(top_k_);
        if (soc_b200_topk(model_, 0, static_cast<int>(top_k_), result->top_logits.data(), ids.data()) != SOC_B200_OK)
            return Fail(soc_b200_last_error(), error_message);
        result->top_token_ids.assign(ids.begin(), ids.end());
        running_token_ids_.push_back(next);
        return true;
    }

    // generation_context.cpp:118-172, with the decode loop resident on the device.
    bool Generate(const std::vector<int>& prompt_token_ids, std::size_t max_new_tokens, int eos_token_id,
                  std::vector<int>* generated_token_ids, std::string* error_message) {
        if (generated_token_ids == nullptr)
            return Fail("GenerationContext generate requires a non-null generated_token_ids output", error_message);
        generated_token_ids->clear();
        if (prompt_token_ids.empty()) return Fail("GenerationContext prefill requires at least one token", error_message);
        if (prompt_token_ids.size() + (max_new_tokens ? max_new_tokens - 1 : 0) > max_sequence_length_)
            return Fail("GenerationContext sequence length would exceed max_sequence_length", error_message);
        Reset();
        std::vector<int32_t> ids(prompt_token_ids.begin(), prompt_token_ids.end());
        std::vector<int32_t> out(max_new_tokens ? max_new_tokens : 1);
        int n = 0;
        if (soc_b200_generate(model_, kv_, seq_, ids.data(), static_cast<int>(ids.size()),
                              static_cast<int>(max_new_tokens), eos_token_id, out.data(), &n) != SOC_B200_OK)
            return Fail(soc_b200_last_error(), error_message);
        generated_token_ids->assign(out.begin(), out.begin() + n);
        prompt_token_ids_ = prompt_token_ids;
        running_token_ids_ = prompt_token_ids;
        running_token_ids_.insert(running_token_ids_.end(), generated_token_ids->begin(), generated_token_ids->end());
        return true;
    }

    // generation_context.cpp:174-179
    void Reset() {
        soc_b200_kv_reset(kv_, seq_);
        prompt_token_ids_.clear();
        running_token_ids_.clear();
        prefill_next_ = -1;
    }

    // Greedy id of the prompt's last row after Prefill (the first generated token).
    int prefill_next_token() const { return prefill_next_; }
    // Appends the id picked after Prefill to the running sequence (what Generate does).
    void AcceptPrefillToken() { running_token_ids_.push_back(prefill_next_); }

    const std::vector<int>& prompt_token_ids() const { return prompt_token_ids_; }
    const std::vector<int>& running_token_ids() const { return running_token_ids_; }

private:
    static bool Fail(const char* msg, std::string* error_message) {
        if (error_message != nullptr) *error_message = msg;
        return false;
    }

    soc_model* model_;
    soc_kv* kv_;
    int seq_;
    std::size_t max_sequence_length_;
    std::size_t top_k_ = 1;
    soc_model_info info_{};
    std::vector<int> prompt_token_ids_;
    std::vector<int> running_token_ids_;
    int prefill_next_ = -1;
};

struct ChatMessage {
    std::string role;
    std::string content;
};

// The bundle's tokenizer (host only).  Move-only owner of a soc_tokenizer.
class Tokenizer {
public:
    // TokenizerRuntimeLoader::LoadFromFile + ValidateTokenizerRuntime.
    static Tokenizer LoadFromFile(const std::string& tokenizer_runtime_path) {
        soc_tokenizer* t = nullptr;
        Check(soc_b200_tokenizer_load(tokenizer_runtime_path.c_str(), &t));
        return Tokenizer(t);
    }
    // The tokenizer a manifest names (its path resolved against the manifest's directory).
    static Tokenizer LoadFromManifest(const std::string& manifest_path) {
        std::size_t n = 0;
        soc_b200_manifest_tokenizer_path(manifest_path.c_str(), nullptr, 0, &n);
        std::string path(n + 1, '\0');
        Check(soc_b200_manifest_tokenizer_path(manifest_path.c_str(), &path[0], path.size(), &n));
        path.resize(n);
        return LoadFromFile(path);
    }
    Tokenizer(Tokenizer&& o) noexcept : t_(std::exchange(o.t_, nullptr)) {}
    Tokenizer& operator=(Tokenizer&& o) noexcept {
        std::swap(t_, o.t_);
        return *this;
    }
    Tokenizer(const Tokenizer&) = delete;
    Tokenizer& operator=(const Tokenizer&) = delete;
    ~Tokenizer() { soc_b200_tokenizer_free(t_); }

    std::vector<int> Encode(const std::string& text) const {
        std::vector<int32_t> ids(text.size() + 16);
        int n = 0;
        int rc = soc_b200_tokenizer_encode(t_, text.data(), text.size(), ids.data(), static_cast<int>(ids.size()), &n);
        if (rc == SOC_B200_ERR_CAPACITY) {
            ids.resize(static_cast<std::size_t>(n));
            rc = soc_b200_tokenizer_encode(t_, text.data(), text.size(), ids.data(), n, &n);
        }
        Check(rc);
        return std::vector<int>(ids.begin(), ids.begin() + n);
    }
    std::string Decode(const std::vector<int>& token_ids) const {
        std::vector<int32_t> ids(token_ids.begin(), token_ids.end());
        std::string out(64 + 16 * ids.size(), '\0');
        std::size_t n = 0;
        int rc = soc_b200_tokenizer_decode(t_, ids.data(), static_cast<int>(ids.size()), &out[0], out.size(), &n);
        if (rc == SOC_B200_ERR_CAPACITY) {
            out.assign(n, '\0');
            rc = soc_b200_tokenizer_decode(t_, ids.data(), static_cast<int>(ids.size()), &out[0], out.size(), &n);
        }
        Check(rc);
        out.resize(n);
        return out;
    }
    // Qwen3TemplateBuilder::BuildPrompt.
    std::string BuildPrompt(const std::vector<ChatMessage>& messages, bool add_generation_prompt, bool enable_thinking,
                            const std::string& system_prompt_override = "") const {
        std::vector<const char*> roles, contents;
        std::size_t cap = 256 + system_prompt_override.size();
        for (const ChatMessage& m : messages) {
            roles.push_back(m.role.c_str());
            contents.push_back(m.content.c_str());
            cap += m.role.size() + m.content.size() + 32;
        }
        std::string out(cap, '\0');
        std::size_t n = 0;
        auto call = [&] {
            return soc_b200_chat_prompt(t_, roles.data(), contents.data(), static_cast<int>(messages.size()),
                                        add_generation_prompt, enable_thinking, system_prompt_override.c_str(), &out[0],
                                        out.size(), &n);
        };
        int rc = call();
        if (rc == SOC_B200_ERR_CAPACITY) {
            out.assign(n, '\0');
            rc = call();
        }
        Check(rc);
        out.resize(n);
        return out;
    }
    // StartupValidator::ValidateManifestAndTokenizer's vocab checks against a loaded model.
    void CheckModel(const soc_model_info& info) const { Check(soc_b200_tokenizer_check_model(t_, info.vocab)); }
    const soc_tokenizer* handle() const { return t_; }

private:
    explicit Tokenizer(soc_tokenizer* t) : t_(t) {}
    static void Check(int rc) {
        if (rc != SOC_B200_OK) throw std::runtime_error(soc_b200_last_error());
    }
    soc_tokenizer* t_ = nullptr;
};

// RuntimeGenerationOptions from the manifest's generation_config (defaults where absent).
inline soc_generation_options GenerationOptionsFromManifest(const std::string& manifest_path) {
    soc_generation_options o{};
    if (soc_b200_manifest_generation_options(manifest_path.c_str(), &o) != SOC_B200_OK)
        throw std::runtime_error(soc_b200_last_error());
    return o;
}

}  // namespace soc::b200
