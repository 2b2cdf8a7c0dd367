// Persistent batch-1 decode kernel (decode_mk.cu): one cooperative launch runs
// `steps` greedy decode steps of one sequence through every layer and the lm_head.
#pragma once

#include "common.cuh"

namespace socb {

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
    int wfmt;  // WF_F16 / WF_BF16 for the block linears and the embedding/lm_head
    const MKLayer* layers;  // device array [L]
    const void* embed;
    const void* lm_head;
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
    // activation vectors shared between CTAs
    float* h;                 // [H] residual stream
    float* qkv;               // [(hq + 2 hkv) D]
    float* attn;              // [hq D]
    float* act;               // [I]
    float* att_part;          // [hkv][splits][G][D + 2] split-K partials
    unsigned int* flags;      // [mk_flag_count(L, hkv, grid)] phase flags, zeroed before launch
    unsigned long long* best; // [steps][grid] per-CTA argmax keys
    int* err;
    int att_splits;
    // optional phase trace of the first step (nullptr = off): %globaltimer stamps,
    // [grid][mk_trace_stride(L)]; slots in decode_mk.cu
    unsigned long long* trace;
};

constexpr int MK_TRACE_PER_LAYER = 16;
constexpr int MK_TRACE_CHUNKS = 64;  // + per CTA: issue, consumer-arrival and ready stamps of the first 64 chunks
__host__ __device__ inline size_t mk_trace_stride(int L) { return static_cast<size_t>(L + 1) * MK_TRACE_PER_LAYER + 3 * MK_TRACE_CHUNKS; }

int mk_flag_count(int L, int hkv, int grid);
// Floats of the four shared activation vectors (h, qkv, attn, act), in that order.
size_t mk_vec_floats(int H, int I, int hq, int hkv, int D);
// Whether the persistent kernel supports this shape on a grid of `grid` CTAs.
bool mk_supported(int H, int I, int hq, int hkv, int D, int wfmt, int grid);
int mk_grid(int device);
void mk_launch(const MKParams& p, int grid, cudaStream_t st);

}  // namespace socb
