// TEST INFRASTRUCTURE ONLY -- a C-ABI shim over the reference CPU runtime.
//
// Linked with the reference's own sources (SongWooYoung/SoC Mac/cpu/src/*.cpp,
// compiled unchanged by oracle/Makefile) into oracle/_ref/libsocref.so.  It
// lets the tests pin the C oracle against the real reference, and bench.py
// time the reference as the CPU baseline.  It calls exactly what the
// reference's GPU regression harness calls: QwenModelLoader::LoadModel and
// QwenCausalLM::ForwardLogitsCached (Mac/cpu/src/qwen_causal_lm.cpp:74-80),
// never GenerationSession::Generate (which runs the prompt twice,
// Mac/cpu/src/generation_session.cpp:55-56).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "header/grouped_query_attention.h"
#include "header/kv_cache.h"
#include "header/linear.h"
#include "header/qwen_causal_lm.h"
#include "header/qwen_model_loader.h"
#include "header/rms_norm_module.h"
#include "header/rope.h"
#include "header/runtime_assets.h"
#include "header/runtime_pipeline.h"
#include "header/sampler.h"
#include "header/startup_validator.h"
#include "header/tokenizer_runtime.h"

namespace {
thread_local std::string g_err;

struct RefModel {
    std::unique_ptr<QwenCausalLM> model;
    std::size_t vocab = 0, layers = 0, kv_heads = 0, head_dim = 0;
};

int Fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}

Tensor Int32Tensor(const int32_t* ids, int n) {
    return Tensor(Storage::FromOwnedCopy(ids, sizeof(int32_t) * static_cast<std::size_t>(n)), DType::Int32,
                  {1, static_cast<std::size_t>(n)});
}

Tensor FloatTensor(const float* v, const std::vector<std::size_t>& shape) {
    std::size_t n = 1;
    for (auto s : shape) n *= s;
    return Tensor(Storage::FromOwnedCopy(v, sizeof(float) * n), DType::Float32, shape);
}
}  // namespace

extern "C" {

const char* socref_last_error() { return g_err.c_str(); }

void* socref_load(const char* manifest_path) {
    try {
        const ManifestData manifest = ManifestLoader::LoadFromFile(manifest_path);
        const Qwen3Config cfg = StartupValidator::ValidateManifest(manifest);
        auto* m = new RefModel();
        m->model = std::make_unique<QwenCausalLM>(QwenModelLoader::LoadModel(manifest));
        m->vocab = cfg.vocab_size;
        m->layers = cfg.num_hidden_layers;
        m->kv_heads = cfg.num_key_value_heads;
        m->head_dim = cfg.head_dim;
        return m;
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void socref_free(void* p) { delete static_cast<RefModel*>(p); }

// RuntimePipeline::LoadBundle (manifest, tokenizer, their validation, the model's tensors):
// 0, or -1 with the reference's message in socref_last_error.
int socref_load_bundle(const char* manifest_path) {
    try {
        const RuntimeBundle bundle = RuntimePipeline::LoadBundle(manifest_path);
        (void)bundle;
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

void* socref_cache_new(void* p, int max_seq) {
    try {
        auto* m = static_cast<RefModel*>(p);
        return new TensorKVCache(m->layers, 1, m->kv_heads, m->head_dim, static_cast<std::size_t>(max_seq));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void socref_cache_free(void* c) { delete static_cast<TensorKVCache*>(c); }

int socref_cache_length(void* c) { return static_cast<int>(static_cast<TensorKVCache*>(c)->length(0)); }

// logits: [n, vocab] floats for every row of the forward (the reference computes all of them).
int socref_forward_cached(void* p, void* c, const int32_t* ids, int n, int pos, float* logits) {
    try {
        auto* m = static_cast<RefModel*>(p);
        const Tensor out = m->model->ForwardLogitsCached(Int32Tensor(ids, n), *static_cast<TensorKVCache*>(c),
                                                         static_cast<std::size_t>(pos));
        if (logits) std::memcpy(logits, out.data<const float>(), sizeof(float) * out.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

// Greedy id of the last row through the reference Sampler (top_k = 1, temperature 1).
int socref_sample_greedy(const float* logits_row, int vocab) {
    const Sampler sampler(SamplerConfig{1.0f, 1});
    return sampler.SampleFromLogits(FloatTensor(logits_row, {1, 1, static_cast<std::size_t>(vocab)}), 0, 0);
}

// The reference Sampler with an explicit config; -1 (message in socref_last_error) when the
// config is rejected.
int socref_sample(const float* logits_row, int vocab, float temperature, int top_k) {
    try {
        const Sampler sampler(SamplerConfig{temperature, static_cast<std::size_t>(top_k)});
        return sampler.SampleFromLogits(FloatTensor(logits_row, {1, 1, static_cast<std::size_t>(vocab)}), 0, 0);
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

// KV rows [start, end) of one layer, as TensorKVCache::Read returns them ([S, Hkv, D] fp32).
int socref_kv_read(void* c, int layer, int start, int end, float* k, float* v) {
    try {
        const auto kv = static_cast<TensorKVCache*>(c)->Read(static_cast<std::size_t>(layer), 0,
                                                             static_cast<std::size_t>(start),
                                                             static_cast<std::size_t>(end));
        std::memcpy(k, kv.first.data<const float>(), sizeof(float) * kv.first.numel());
        std::memcpy(v, kv.second.data<const float>(), sizeof(float) * kv.second.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

// ---- module-level entry points (for pinning the C restatement op by op) ----

int socref_linear(const float* x, int rows, int in, const float* w, int out, float* y) {
    try {
        const Linear lin(FloatTensor(w, {static_cast<std::size_t>(out), static_cast<std::size_t>(in)}));
        const Tensor r = lin.Forward(FloatTensor(x, {static_cast<std::size_t>(rows), static_cast<std::size_t>(in)}));
        std::memcpy(y, r.data<const float>(), sizeof(float) * r.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

int socref_rmsnorm(const float* x, int rows, int n, const float* w, float eps, float* y) {
    try {
        const RMSNormModule norm(FloatTensor(w, {static_cast<std::size_t>(n)}), eps);
        const Tensor r = norm.Forward(FloatTensor(x, {static_cast<std::size_t>(rows), static_cast<std::size_t>(n)}));
        std::memcpy(y, r.data<const float>(), sizeof(float) * r.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

int socref_rope(float* x, int T, int heads, int D, double theta, int pos0) {
    try {
        const RoPE rope(static_cast<std::size_t>(D), theta);
        Tensor t = FloatTensor(x, {1, static_cast<std::size_t>(T), static_cast<std::size_t>(heads), static_cast<std::size_t>(D)});
        rope.ApplyInPlace(t, static_cast<std::size_t>(pos0));
        const Tensor& tc = t;
        std::memcpy(x, tc.data<const float>(), sizeof(float) * tc.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

int socref_attention(const float* q, int T, int Hq, const float* k, const float* v, int S, int Hkv, int D, int prefix,
                     float* out) {
    try {
        const GroupedQueryAttention att(static_cast<std::size_t>(Hq), static_cast<std::size_t>(Hkv),
                                        static_cast<std::size_t>(D), true);
        const auto sz = [](int a) { return static_cast<std::size_t>(a); };
        const Tensor r = att.ForwardWithPrefix(FloatTensor(q, {1, sz(T), sz(Hq), sz(D)}),
                                               FloatTensor(k, {1, sz(S), sz(Hkv), sz(D)}),
                                               FloatTensor(v, {1, sz(S), sz(Hkv), sz(D)}), sz(prefix));
        std::memcpy(out, r.data<const float>(), sizeof(float) * r.numel());
        return 0;
    } catch (const std::exception& e) {
        return Fail(e);
    }
}


// ---- tokenizer / chat template (TokenizerRuntimeLoader::LoadFromFile, runtime_assets.cpp:170-216;
// TokenizerRuntime::{Encode, Decode}, tokenizer_runtime.cpp; Qwen3TemplateBuilder::BuildPrompt,
// runtime_assets.cpp:221-258)
void* socref_tokenizer_load(const char* path) {
    try {
        TokenizerRuntimeData data = TokenizerRuntimeLoader::LoadFromFile(path);
        StartupValidator::ValidateTokenizerRuntime(data);
        return new TokenizerRuntime(std::move(data));
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void socref_tokenizer_free(void* t) { delete static_cast<TokenizerRuntime*>(t); }

int socref_tokenizer_encode(void* t, const char* text, int len, int32_t* ids, int cap) {
    try {
        const std::vector<int> out = static_cast<TokenizerRuntime*>(t)->Encode(std::string(text, len));
        for (int i = 0; i < static_cast<int>(out.size()) && i < cap; ++i) ids[i] = out[i];
        return static_cast<int>(out.size());
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

int socref_tokenizer_decode(void* t, const int32_t* ids, int n, char* out, int cap) {
    try {
        const std::string s = static_cast<TokenizerRuntime*>(t)->Decode(std::vector<int>(ids, ids + n));
        std::memcpy(out, s.data(), std::min<std::size_t>(s.size(), static_cast<std::size_t>(cap)));
        return static_cast<int>(s.size());
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

int socref_chat_prompt(void* t, const char* user, int add_generation_prompt, int enable_thinking,
                       const char* system_override, char* out, int cap) {
    try {
        const Qwen3TemplateBuilder builder(static_cast<TokenizerRuntime*>(t)->runtime_data().template_runtime);
        const std::string s = builder.BuildPrompt(std::vector<ChatMessage>{{"user", user}}, add_generation_prompt != 0,
                                                  enable_thinking != 0, system_override ? system_override : "");
        std::memcpy(out, s.data(), std::min<std::size_t>(s.size(), static_cast<std::size_t>(cap)));
        return static_cast<int>(s.size());
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

// Qwen3TemplateBuilder::BuildPrompt over n (role, content) messages.
int socref_chat_prompt_messages(void* t, const char* const* roles, const char* const* contents, int n,
                                int add_generation_prompt, int enable_thinking, const char* system_override, char* out,
                                int cap) {
    try {
        const Qwen3TemplateBuilder builder(static_cast<TokenizerRuntime*>(t)->runtime_data().template_runtime);
        std::vector<ChatMessage> messages;
        for (int i = 0; i < n; ++i) messages.push_back(ChatMessage{roles[i], contents[i]});
        const std::string s = builder.BuildPrompt(messages, add_generation_prompt != 0, enable_thinking != 0,
                                                  system_override ? system_override : "");
        std::memcpy(out, s.data(), std::min<std::size_t>(s.size(), static_cast<std::size_t>(cap)));
        return static_cast<int>(s.size());
    } catch (const std::exception& e) {
        return Fail(e);
    }
}

}  // extern "C"
