// Host launchers of the modular Qwen3 kernels (kernels.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace socb {

// Number of kernels this library has launched (graph replays add their kernel count).
void count_launches(long long n);
long long launches_so_far();

// Paged KV cache view of one layer: pool [pages][kv_heads][page_tokens][head_dim] fp16.
struct KVLayerView {
    __half* k;
    __half* v;
    const int* page_table;  // [max_seqs][max_pages]
    int max_pages;
    int page_tokens;
    // optional 2-D TMA views of the whole K / V pools ([rows = L * pages * hkv * 16, head_dim],
    // 64 x 16 boxes, 128-byte swizzle) and this layer's first row; null when not built
    const CUtensorMap* tmk = nullptr;
    const CUtensorMap* tmv = nullptr;
    int row0 = 0;
};

// Per-forward row descriptors (one row = one token of some sequence), all device pointers.
struct Rows {
    const int* tokens;  // [n]
    const int* seq;     // [n]
    const int* pos;     // [n] absolute position of the row's token
    int n;
};

void launch_embed(int wfmt, const void* table, int hidden, int vocab, const int* tokens, int rows, float* h,
                  int* err, cudaStream_t st);

// y[r, o] (mode)= sum_i x'[r, i] * W[o, i], x' = rmsnorm(x[r], norm_w) when norm_w != nullptr.
void launch_linear(int wfmt, const void* W, const void* scales, int out_f, int in_f, const float* x, int ldx,
                   int rows, const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st);

// Tensor-core variant for fp16 / int8 g64 / int4 g32 weights and up to 16 input rows per
// row block (linear_mma.cu); false when the shape or format is outside it (launch_linear then
// runs the CUDA-core GEMV).  SOC_B200_LINEAR_MMA=0 turns it off.
bool launch_linear_mma(int wfmt, const void* W, const void* scales, int out_f, int in_f, const float* x, int ldx,
                       int rows, const float* norm_w, float eps, float* y, int ldy, int mode, cudaStream_t st);

void launch_qk_norm_rope_kv(const float* qkv, const Rows& rows, int hq, int hkv, int head_dim, const float* qn_w,
                            const float* kn_w, float eps, const float2* rope_cs, int rope_len, const KVLayerView& kv,
                            float* q_out, int* err, cudaStream_t st);

// Causal GQA over the paged cache; visible keys of a row = [0, pos], cut into `splits` key ranges
// (computed per row on the device).  `scratch` (may be null when splits == 1) holds the split-K
// partials: rows*hq*splits*(head_dim + 2) floats.
void launch_attention(const float* q, const Rows& rows, int splits, int hq, int hkv, int head_dim,
                      const KVLayerView& kv, float* out, float* scratch, size_t scratch_floats, int* err,
                      cudaStream_t st);
// Page-streaming variant (attn_decode.cu) used by launch_attention; false when the shape is
// outside its instances (16-token pages, head_dim 64/128, 1/2/4/8 query heads per kv head).
bool launch_attention_pages(const float* q, const Rows& rows, int splits, int hq, int hkv, int head_dim,
                            const KVLayerView& kv, float* out, float* scratch, int* err, cudaStream_t st);
int attention_splits(int rows, int hkv, int max_visible);

// Causal attention of the n rows of one prefill chunk (row r = position start + r of
// sequence `seq`) on tensor cores (attn_prefill.cu).  Same output layout as launch_attention.
void launch_flash_prefill(const float* q, int n, int hq, int hkv, int head_dim, int seq, int start,
                          const KVLayerView& kv, float* out, cudaStream_t st);
// The same attention on tcgen05 with S and O in tensor memory (attn_prefill_tc.cu); needs the
// cache's TMA maps.  Not yet used by the forward path.
void launch_flash_prefill_tc(const float* q, int n, int hq, int hkv, int head_dim, int seq, int start,
                             const KVLayerView& kv, float* out, int* err, cudaStream_t st);

// Seeded pseudo-random K and V (about N(0, 1), fp16) for positions [0, n_tokens) of sequence
// `seq` in every layer; `pages` = that sequence's page-table row.
// hkv = kv heads held here, heads [head_off, head_off + hkv) of hkv_total (tensor parallelism).
void launch_kv_fill_random(__half* kpool, __half* vpool, size_t layer_stride, const int* pages, int page_tokens,
                           int hkv, int hkv_total, int head_off, int D, int L, int n_tokens, int seq,
                           unsigned long long seed, cudaStream_t st);

// temperature: the pick maximises logit / temperature (IEEE single division; 1 = the logits).
// `keys` is scratch for one 64-bit key per row.
void launch_argmax(const float* logits, int vocab, int ld, int rows, float temperature, unsigned long long* keys,
                   int* next_ids, cudaStream_t st);
// Vocab-parallel greedy pick: per-row (value, global index) keys of one shard, and the merge
// of all shards' keys [shards][rows] (lowest global index wins ties, as above).
void launch_argmax_keys(const float* logits, int vocab, int ld, int rows, int v_off, float temperature, unsigned long long* keys,
                        cudaStream_t st);
void launch_argmax_merge(const unsigned long long* keys_all, int shards, int rows, int* next_ids, cudaStream_t st);
// Top-k candidates of one logits row (k <= TOPK_MAX); element g at base + (g / seg_len) * seg_stride
// + g % seg_len.  `cand` holds topk_scratch_keys(V, k) keys; outputs are device arrays of k.
constexpr int TOPK_MAX = 64;
int topk_scratch_keys(int V, int k);
void launch_topk(const float* base, int V, int seg_len, size_t seg_stride, float temperature, int k,
                 unsigned long long* cand, float* top_logits, int* top_ids, cudaStream_t st);

void launch_rmsnorm(const float* x, int rows, int n, const float* w, float eps, float* y, cudaStream_t st);

}  // namespace socb
