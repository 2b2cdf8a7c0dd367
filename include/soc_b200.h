/*
 * soc_b200 -- C ABI of the B200-native Qwen3 forward path.
 *
 * Drop-in boundary for the reference runtime's hot path (SongWooYoung/SoC):
 * the entry points below replace, one for one, what a host runtime calls on
 * the reference's model objects.  Plain pointers and sizes only; every call
 * returns 0 (SOC_B200_OK) or a negative status, with a thread-local message
 * in soc_b200_last_error() (the reference throws std::runtime_error, e.g.
 * Mac/cpu/src/linear.cpp:9-11, or returns bool + std::string*,
 * Mac/gpu/src/runtime/generation_context.cpp:97-101).
 *
 * Ownership: the library owns all device memory it allocates; host buffers
 * passed in are copied before the call returns.  Threading: one CUDA stream
 * per context; calls on one context (and on the models and caches made from
 * it) must be serialised by the caller, as with the reference's
 * GenerationContext (not thread-safe).
 */
#ifndef SOC_B200_H
#define SOC_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SOC_B200_API __attribute__((visibility("default")))
#else
#define SOC_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SOC_B200_OK 0
#define SOC_B200_ERR_INVALID (-1)   /* bad argument, shape or state */
#define SOC_B200_ERR_CUDA (-2)      /* CUDA runtime failure */
#define SOC_B200_ERR_IO (-3)        /* file missing / short */
#define SOC_B200_ERR_FORMAT (-4)    /* manifest or tensor record rejected */
#define SOC_B200_ERR_CAPACITY (-5)  /* KV cache or workspace exhausted */
#define SOC_B200_ERR_RANGE (-6)     /* token id outside [0, vocab) */
#define SOC_B200_ERR_DEVICE (-7)    /* a kernel reported an error status */

/* Weight formats for soc_b200_load_bundle / soc_b200_linear. */
#define SOC_B200_WEIGHTS_NATIVE 0   /* whatever the bundle stores */
#define SOC_B200_WEIGHTS_F16 1
#define SOC_B200_WEIGHTS_BF16 2
#define SOC_B200_WEIGHTS_INT8_G64 3 /* group 64 along in_features, fp16 scales */
#define SOC_B200_WEIGHTS_INT4_G32 4 /* group 32, two per byte (low nibble first), fp16 scales */

typedef struct soc_ctx soc_ctx;
typedef struct soc_model soc_model;
typedef struct soc_kv soc_kv;

typedef struct {
    int layers, hidden, intermediate, q_heads, kv_heads, head_dim, vocab;
    int tied_embeddings;   /* lm_head aliases the embedding table */
    int weight_format;     /* SOC_B200_WEIGHTS_* of the block linears */
    int max_position;      /* rows of the RoPE table */
    float rms_norm_eps;
    double rope_theta;
    int tp_rank;           /* tensor-parallel rank of this shard (0 without tensor parallelism) */
    int tp_size;           /* ranks sharing the model (1 without tensor parallelism); the head,
                              intermediate and vocab counts above are the whole model's */
} soc_model_info;

/* Message of the last failed call on this thread ("" if none). */
SOC_B200_API const char* soc_b200_last_error(void);

/* Kernels launched by this library in this process so far (a CUDA-graph
 * replay counts every kernel node).  No counterpart in the reference, which
 * has no device kernels; used to attribute device work in benchmarks. */
SOC_B200_API long long soc_b200_kernel_launches(void);

/* Open device `device` (one stream).  Replaces MetalContext::CreateDefault
 * (Mac/gpu/src/metal/metal_context.mm:78). */
SOC_B200_API int soc_b200_open(int device, soc_ctx** out);
SOC_B200_API void soc_b200_close(soc_ctx* ctx);
/* Wait for all work queued on the context's stream. */
SOC_B200_API int soc_b200_synchronize(soc_ctx* ctx);
/* The context's cudaStream_t (for event timing by the caller). */
SOC_B200_API void* soc_b200_stream(soc_ctx* ctx);

/* Load a soc.cpp.llm_export v2 bundle into device memory.  Validation and
 * error text follow ManifestLoader::LoadFromFile + StartupValidator::
 * ValidateManifest + QwenModelLoader::LoadModel (Mac/cpu/src/runtime_assets.cpp:
 * 138-168, startup_validator.cpp:5-23, qwen_model_loader.cpp:35-93) and
 * WeightLoader::LoadTensor (weight_loader.cpp:17-30).  Without tensor
 * parallelism tp_rank = 0, tp_size = 1, nccl_comm = NULL.  With tp_size > 1 this
 * rank keeps heads [tp_rank * hq / tp_size, ...) of q (and the matching kv heads),
 * rows of gate/up and columns of o_proj/down_proj, and vocab rows [tp_rank * V /
 * tp_size, ...) of the lm_head; nccl_comm is that group's ncclComm_t
 * (soc_b200_nccl_comm_create or the caller's own); the KV cache then holds the
 * local kv heads. */
SOC_B200_API int soc_b200_load_bundle(soc_ctx* ctx, const char* manifest_path, int weight_format, int tp_rank, int tp_size,
                         void* nccl_comm, soc_model** out);
SOC_B200_API int soc_b200_model_info(const soc_model* model, soc_model_info* out);
/* The checks RuntimePipeline::LoadBundle makes before it has a model (Mac/cpu/src/
 * runtime_pipeline.cpp:36-41): the manifest and tokenizer loaders, StartupValidator::
 * ValidateManifestAndTokenizer (startup_validator.cpp:5-23, 77-101) and the record checks of
 * every tensor QwenModelLoader::LoadModel reads (qwen_model_loader.cpp:35-93, weight_loader.cpp:
 * 17-30), with the same messages.  Host only: needs no device and reads no weight data (tensor
 * files are only measured), so a host can reject a broken bundle before it opens a GPU. */
SOC_B200_API int soc_b200_validate_bundle(const char* manifest_path);
/* Sampler(SamplerConfig) (Mac/cpu/src/sampler.cpp:17-57) for every later next-token pick
 * of this model (prefill, decode, generate, decode_noalloc): the id maximising
 * logit / temperature, the division IEEE single precision as in the reference, lowest id on
 * ties.  The reference returns the best of the top_k largest such scores, which is that
 * maximum for every top_k >= 1, so top_k is only validated.  One difference: when the
 * largest score repeats and top_k > 1, the reference returns whichever of the tied ids its
 * C++ library's partial_sort puts first (not specified by the language; the lowest id for
 * top_k = 1), this library the lowest.  Defaults: 1.0 and 1; the argument checks and their
 * messages are the reference's. */
SOC_B200_API int soc_b200_set_sampler(soc_model* model, float temperature, size_t top_k);
SOC_B200_API void soc_b200_free_model(soc_model* model);


/* Paged fp16 KV cache for up to max_seqs sequences and max_tokens cached
 * tokens in total, page_tokens per page (16).  Replaces TensorKVCache
 * (Mac/cpu/src/kv_cache.cpp:20-44) and the Metal KVCache::CreateShared. */
SOC_B200_API int soc_b200_kv_create(soc_model* model, int max_seqs, int max_tokens, int page_tokens, soc_kv** out);
SOC_B200_API void soc_b200_free_kv(soc_kv* kv);
/* Drop a sequence's cached tokens (TensorKVCache::ClearSequence, kv_cache.cpp:112-115). */
SOC_B200_API int soc_b200_kv_reset(soc_kv* kv, int seq);
/* Cached length of a sequence (TensorKVCache::length), or a negative status. */
SOC_B200_API int soc_b200_kv_length(const soc_kv* kv, int seq);
/* Positions [start, end) of one layer as float32 [end-start, kv_heads, head_dim]
 * K and V (TensorKVCache::Read, kv_cache.cpp:80-110). */
SOC_B200_API int soc_b200_kv_read(soc_kv* kv, int seq, int layer, int start, int end, float* k, float* v);
/* Write positions [start, end) of one layer from float32 host rows (rounded to
 * fp16); extends the sequence length to `end` (TensorKVCache::Write, kv_cache.cpp:50-78). */
SOC_B200_API int soc_b200_kv_write(soc_kv* kv, int seq, int layer, int start, int end, const float* k, const float* v);

/* Benchmark and test helper; it has no counterpart in the reference.  Replaces sequence
 * `seq` of the cache by n_tokens positions whose K and V (every layer and kv head) are
 * seeded pseudo-random values of about N(0, 1) rounded to fp16: element e = (pos * kv_heads
 * + head) * head_dim + d of stream s = (seq * layers + layer) * 2 + (0 for K, 1 for V) is
 * sum / 65536 - 6, where sum adds the twelve 16-bit fields of splitmix64 outputs at
 * x, x + 1, x + 2 with x = seed + s * 0xD1B54A32D192ED03 + 3 e (all arithmetic mod 2^64).
 * Queued on the context stream without a host synchronisation. */
SOC_B200_API int soc_b200_kv_fill_random(soc_kv* kv, int seq, int n_tokens, unsigned long long seed);

/* Append n tokens to sequence `seq` at its current length and run them
 * through the model (QwenCausalLM::ForwardLogitsCached with position_offset =
 * cached length, Mac/cpu/src/qwen_causal_lm.cpp:74-80).  logits_last (nullable)
 * receives the vocab logits of the last token; next_id (nullable) its greedy
 * id (Sampler::SampleFromLogits, top_k 1). */
SOC_B200_API int soc_b200_prefill(soc_model* model, soc_kv* kv, int seq, const int32_t* ids, int n, float* logits_last,
                     int32_t* next_id);

/* One decode step for n_seqs distinct sequences, each appending last_ids[i]
 * (GenerationContext::DecodeNextToken, Mac/gpu/src/runtime/generation_context.cpp:
 * 61-116, batched and ragged).  logits (nullable) receives [n_seqs, vocab]. */
SOC_B200_API int soc_b200_decode(soc_model* model, soc_kv* kv, int n_seqs, const int* seq_ids, const int32_t* last_ids,
                    float* logits, int32_t* next_ids);

/* Reset `seq`, prefill the prompt and decode greedily up to max_new tokens,
 * stopping after eos_token_id when it is >= 0 (GenerationContext::Generate,
 * generation_context.cpp:118-172).  out_ids must hold max_new ids; *n_out
 * receives the count.  The decode steps run back to back on the device; with the
 * persistent batch-1 decode kernel the eos stop happens on the device (no step after
 * it runs), elsewhere the steps after it are computed and dropped. */
SOC_B200_API int soc_b200_generate(soc_model* model, soc_kv* kv, int seq, const int32_t* prompt, int n_prompt, int max_new,
                      int eos_token_id, int32_t* out_ids, int* n_out);

/* As soc_b200_generate with DEVICE pointers for the prompt and the max_new
 * output ids, no EOS stop and no host synchronisation (work is queued on the
 * context stream). */
SOC_B200_API int soc_b200_generate_device(soc_model* model, soc_kv* kv, int seq, const int32_t* d_prompt, int n_prompt,
                             int max_new, int32_t* d_out);

/* ---- string pipeline (host only, no GPU) ----------------------------------
 * The bundle's tokenizer (tokenizer/tokenizer_runtime.json) and the Qwen3 chat
 * template.  Replaces TokenizerRuntimeLoader::LoadFromFile + StartupValidator::
 * ValidateTokenizerRuntime (Mac/cpu/src/runtime_assets.cpp:170-216,
 * startup_validator.cpp:25-73), TokenizerRuntime::Encode / Decode
 * (Mac/cpu/header/tokenizer_runtime.h:17-18) and Qwen3TemplateBuilder::BuildPrompt
 * (Mac/cpu/src/runtime_assets.cpp:221-258); same results and error texts. */
typedef struct soc_tokenizer soc_tokenizer;
SOC_B200_API int soc_b200_tokenizer_load(const char* tokenizer_runtime_path, soc_tokenizer** out);
SOC_B200_API void soc_b200_tokenizer_free(soc_tokenizer* tokenizer);
/* *n_ids = number of ids; SOC_B200_ERR_CAPACITY (first `capacity` ids written) when larger. */
SOC_B200_API int soc_b200_tokenizer_encode(const soc_tokenizer* tokenizer, const char* text, size_t len, int32_t* ids,
                                           int capacity, int* n_ids);
/* *len = bytes of text (not NUL-terminated); SOC_B200_ERR_CAPACITY when larger than capacity. */
SOC_B200_API int soc_b200_tokenizer_decode(const soc_tokenizer* tokenizer, const int32_t* ids, int n, char* text,
                                           size_t capacity, size_t* len);
/* Messages (role, content) -> prompt text; without a "system" message the override (or the
 * template's default system prompt) is prepended. */
SOC_B200_API int soc_b200_chat_prompt(const soc_tokenizer* tokenizer, const char* const* roles,
                                      const char* const* contents, int n_messages, int add_generation_prompt,
                                      int enable_thinking, const char* system_prompt_override, char* out,
                                      size_t capacity, size_t* len);

/* StartupValidator::ValidateManifestAndTokenizer's cross checks of a tokenizer against the
 * model's vocab_size (Mac/cpu/src/startup_validator.cpp:77-101). */
SOC_B200_API int soc_b200_tokenizer_check_model(const soc_tokenizer* tokenizer, long long model_vocab_size);

/* RuntimeGenerationOptions (Mac/cpu/header/runtime_pipeline.h:12-17): the defaults, overridden
 * by the manifest's generation_config as RuntimePipeline::GenerationOptionsFromManifest does
 * (Mac/cpu/src/runtime_pipeline.cpp:43-55; "max_length" feeds max_sequence_length). */
typedef struct soc_generation_options {
    size_t max_new_tokens;      /* 32 */
    float temperature;          /* 1.0 */
    size_t top_k;               /* 1 */
    int eos_token_id;           /* -1: disabled */
    size_t max_sequence_length; /* 256: the KV capacity of a generation */
} soc_generation_options;
SOC_B200_API int soc_b200_manifest_generation_options(const char* manifest_path, soc_generation_options* out);
/* The manifest's tokenizer_runtime_file resolved against the manifest's directory
 * (ManifestLoader::LoadFromFile, Mac/cpu/src/runtime_assets.cpp:138-168); NUL-terminated,
 * *len excludes the NUL. */
SOC_B200_API int soc_b200_manifest_tokenizer_path(const char* manifest_path, char* out, size_t capacity, size_t* len);
/* Sampler's argument checks (Mac/cpu/src/sampler.cpp:17-20).  The reference sampler returns
 * the best of the top_k largest logit/temperature scores, which is the greedy argmax the
 * decode kernels compute for every temperature > 0. */
SOC_B200_API int soc_b200_sampler_check(float temperature, size_t top_k);

/* Tensor parallelism plumbing (the reference is single-device; these have no counterpart
 * in it).  NCCL is loaded at run time from libnccl.so.2.  Rank 0 creates the id, every rank
 * receives its 128 bytes out of band and creates the communicator on its own context's
 * device; the communicator is then passed to soc_b200_load_bundle with tp_rank / tp_size.
 * Every rank of a tensor-parallel model must make the same calls in the same order (the
 * forward runs collectives), including the same choice of NULL / non-NULL logits outputs. */
SOC_B200_API int soc_b200_nccl_unique_id(void* id_out /* 128 bytes */);
SOC_B200_API int soc_b200_nccl_comm_create(soc_ctx* ctx, int nranks, int rank, const void* id, void** comm_out);
SOC_B200_API int soc_b200_nccl_comm_destroy(void* comm);

/* Kernel-level linear: y[r, :] = W x[r, :] for r < rows, all DEVICE pointers,
 * W [out_features, in_features] in `weight_format` (scales [out, in/group] fp16
 * for the int formats, else NULL), x [rows, in] fp32, y [rows, out] fp32.
 * Restates Linear::Forward (Mac/cpu/src/linear.cpp:51-84).  stream may be NULL
 * (the context stream). */
SOC_B200_API int soc_b200_linear(soc_ctx* ctx, int weight_format, const void* w, const void* scales, int out_features,
                    int in_features, const float* x, int rows, float* y, void* stream);

/* The sampler's candidate list for row `row` of the logits that the last
 * soc_b200_prefill (row 0) or soc_b200_decode (row = index in the batch) call
 * left on the device: the k (1..64) tokens with the largest logit / temperature,
 * larger first, the lower id first among equal values; top_logits gets their raw
 * logits, top_token_ids their ids (host arrays of k).  Replaces the top_logits /
 * top_token_ids that Sampler::SampleFromLogits fills in GenerationStepResult
 * (Mac/gpu/src/runtime/sampler.cpp:58-68, generation_context.h:17-21).  Not
 * after generate or decode_noalloc (their steps keep no logits).  With tensor
 * parallelism every rank makes the same call (the vocab shards are gathered). */
SOC_B200_API int soc_b200_topk(soc_model* model, int row, int k, float* top_logits, int32_t* top_token_ids);

/* One batch-1 decode step of sequence `seq` that allocates no device memory.
 * No counterpart in the reference.  For callers that cannot call cudaMalloc
 * while serving (an engine that gives the whole GPU to its own pool at
 * start-up, or a latency path that must not take cudaMalloc's implicit device
 * synchronisation).  Same inputs and outputs as soc_b200_decode with one
 * sequence: last_id is appended at the cached length, logits (nullable, host)
 * receives the vocab row, next_id the greedy id.  All scratch of the step lives
 * in one static device array of 4 MiB that every GPU loading this library keeps
 * until exit; a model whose step needs more is rejected with
 * SOC_B200_ERR_CAPACITY, and shapes outside the persistent decode kernel's
 * limits with SOC_B200_ERR_INVALID.  The first call on a device looks up the
 * array's device address, so make it before any stream capture.  Calls share
 * the array: calls whose GPU work overlaps race. */
SOC_B200_API int soc_b200_decode_noalloc(soc_model* model, soc_kv* kv, int seq, int32_t last_id, float* logits,
                                         int32_t* next_id);

#ifdef __cplusplus
}
#endif

#endif /* SOC_B200_H */
