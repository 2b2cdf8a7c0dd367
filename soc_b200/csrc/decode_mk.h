// Persistent batch-1 decode kernel (decode_mk.cu): one cooperative launch runs
// `steps` greedy decode steps of one sequence through every layer and the lm_head.
#pragma once

#include "common.cuh"

namespace socb {

// Weights of one layer in the kernel's tiled layout (mk_tile_matrix): 8-row tiles, each
// tile's bytes contiguous, laid out in mma.sync B-fragment order.
struct MKLayer {
    const void* wqkv;  // [(hq + 2 hkv) * D, H]
    const void* wo;    // [H, hq * D]
    const void* wgu;   // [2 I, H], rows (2j, 2j+1) = (gate_j, up_j)
    const void* wd;    // [H, I]
    const float *in_norm, *post_norm, *q_norm, *k_norm;
};

struct MKParams {
    int L, H, I, hq, hkv, D, V;
    float eps;
    int wfmt;  // block linears: WF_F16 / WF_BF16 / WF_I8G64 / WF_I4G32
    int efmt;  // embedding and lm_head: WF_F16 / WF_BF16
    const MKLayer* layers;  // device array [L]
    const void* embed;      // row-major [V, H] (the embedding lookup)
    const void* lm_tiles;   // the lm_head in the tiled layout
    const float* final_norm;
    const float2* rope_cs;
    int rope_len;
    // paged KV cache
    __half* kpool;
    __half* vpool;
    size_t kv_layer_stride;  // elements per layer
    const int* page_table;   // row of this sequence: [max_pages]
    int page_tokens;
    int max_pages;
    // the steps: step t consumes ids[t] at position start + t and writes ids[t + 1]
    int* ids;
    int start;
    int steps;
    float* logits;  // nullable: [steps, V]
    float temperature;  // the pick maximises logit / temperature (1: the logits)
    int eos;            // >= 0: stop at the top of the first step whose input id is eos
    // Activation vectors shared between CTAs, as 64-bit words {fp32 value, 32-bit tag}.  A word
    // written by phase `ph` of layer l in step t carries mk_tag(tag0, t, l, ph); readers wait
    // for the tag they need, so every hand-off is carried by the data itself.
    unsigned long long* vec;   // [mk_vec_words]: h | qkv | attn | act
    unsigned long long* part;  // [hkv][splits][G][D + 2] split-K attention partials (acc, max, sum)
    unsigned int tag0;         // tags of this launch: tag0 + 1 .. tag0 + mk_tags_per_launch
    unsigned long long* best;  // [steps][grid] per-CTA argmax keys (zero = not yet written)
    int* err;
    int att_splits;
    int att_group;  // query heads per attention unit (mk_att_plan)
    int inflight;  // ring chunks the producer keeps in flight (1 .. ring slots)
    // optional phase trace of the first step (nullptr = off): %globaltimer stamps,
    // [grid][mk_trace_stride(L)]; slots in decode_mk.cu
    unsigned long long* trace;
};

constexpr int MK_TRACE_PER_LAYER = 48;
constexpr int MK_TRACE_CHUNKS = 64;
__host__ __device__ inline size_t mk_trace_stride(int L) { return static_cast<size_t>(L + 1) * MK_TRACE_PER_LAYER + 3 * MK_TRACE_CHUNKS; }

constexpr int MK_PHASES = 5;  // tag phases per layer: qkv, attention, o (h), act, down (h)
// Tags one launch of `steps` steps uses (the host advances tag0 by this much per launch).
inline unsigned long long mk_tags_per_launch(int steps, int L) {
    return static_cast<unsigned long long>(steps) * L * MK_PHASES + 8;
}

// 64-bit words of the shared activation vectors (h, qkv, attn, act), in that order.
size_t mk_vec_words(int H, int I, int hq, int hkv, int D);
// Words of the split-K attention partials for `splits` key splits.
size_t mk_part_words(int hq, int hkv, int D, int splits);
// Key splits of the attention for contexts up to max_ctx on a grid of `grid` CTAs, and the query
// heads per attention unit (*group: 1, or hq / hkv).
int mk_att_plan(int max_ctx, int hq, int hkv, int grid, int* group);
// Whether the persistent kernel supports this shape on a grid of `grid` CTAs.
bool mk_supported(int L, int H, int I, int hq, int hkv, int D, int V, int wfmt, int efmt, int grid);
int mk_grid(int device);
// Bytes of one matrix [rows, K] of format `wfmt` in the tiled layout (rows a multiple of 8).
size_t mk_tiled_bytes(int wfmt, int rows, int K);
// Rewrites a row-major matrix (with its group scales for int8 / int4) into the tiled layout.
void mk_tile_matrix(int wfmt, const void* w, const void* scales, int rows, int K, void* dst, cudaStream_t st);
void mk_launch(const MKParams& p, int grid, cudaStream_t st);

}  // namespace socb
