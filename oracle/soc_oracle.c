/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the Qwen3 forward path.
 *
 * A plain-C restatement of the reference CPU runtime's arithmetic
 * (SongWooYoung/SoC, Mac/cpu/src).  It is the checker that the B200 kernels
 * are compared against; nothing in the soc_b200 product links or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may.
 *
 * Every routine keeps the reference's operation order (sequential fp32
 * accumulation in index order, the same libm calls), so with
 * -ffp-contract=off it reproduces the reference bit for bit; the tests pin
 * that against oracle/_ref (the reference sources compiled unchanged).
 *
 * Weight element types: 0 = float32, 1 = float16, 2 = bfloat16.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

/* ---- a parallel for over independent outputs ------------------------------
 * The linears and the attention split their outputs (rows x features, rows x heads)
 * into contiguous ranges, one per host thread.  Every output keeps its own sequential
 * accumulation, so the results do not depend on the thread count (ORACLE_THREADS, else
 * the online CPUs, at most 64). */
typedef void (*range_fn)(void* ctx, long lo, long hi);
typedef struct {
    range_fn fn;
    void* ctx;
    long lo, hi;
} par_job;

static void* par_run(void* a) {
    par_job* j = (par_job*)a;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static int par_threads(void) {
    const char* e = getenv("ORACLE_THREADS");
    long n = e && *e ? atol(e) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return (int)n;
}

/* fn over [0, n) in one range per thread when the work (n * cost) is large enough. */
static void par_for(long n, long cost, range_fn fn, void* ctx) {
    int nt = par_threads();
    if (n * cost < 4000000L || nt <= 1 || n < 2) {
        fn(ctx, 0, n);
        return;
    }
    if (nt > n) nt = (int)n;
    pthread_t th[64];
    par_job jobs[64];
    int started = 0;
    for (int i = 0; i < nt; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].lo = n * i / nt;
        jobs[i].hi = n * (i + 1) / nt;
    }
    for (int i = 1; i < nt; ++i) {
        if (pthread_create(&th[i], NULL, par_run, &jobs[i]) != 0) break;
        started = i;
    }
    par_run(&jobs[0]);
    for (int i = 1; i <= started; ++i) pthread_join(th[i], NULL);
    for (int i = started + 1; i < nt; ++i) par_run(&jobs[i]); /* threads that could not start */
}

/* IEEE half -> float, exact (restates Float16ToFloat32, Mac/cpu/src/dtype.cpp:76-106). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 0x1fu;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int32_t e = -14;
            while ((mantissa & 0x400u) == 0) { mantissa <<= 1; --e; }
            mantissa &= 0x3ffu;
            bits = sign | ((uint32_t)(e + 127) << 23) | (mantissa << 13);
        }
    } else if (exponent == 0x1fu) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* bfloat16 -> float (Mac/cpu/src/dtype.cpp:108-113). */
static float bf16_to_f32(uint16_t v) {
    uint32_t bits = (uint32_t)v << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Element read of a float-like weight (DTypeReadFloat, Mac/cpu/src/dtype.cpp:165-176). */
static inline float rd(const void* p, int dt, size_t i) {
    switch (dt) {
        case OR_F32: return ((const float*)p)[i];
        case OR_F16: return oracle_f16_to_f32(((const uint16_t*)p)[i]);
        default: return bf16_to_f32(((const uint16_t*)p)[i]);
    }
}

typedef struct {
    const float* x;
    int in, wdt, out;
    const void* w;
    float* y;
} lin_ctx;

static void lin_range(void* c, long lo, long hi) {
    const lin_ctx* a = (const lin_ctx*)c;
    for (long j = lo; j < hi; ++j) {
        const long r = j / a->out, o = j % a->out;
        const float* xr = a->x + (size_t)r * a->in;
        const size_t base = (size_t)o * a->in;
        float v = 0.0f;
        for (int i = 0; i < a->in; ++i) v += xr[i] * rd(a->w, a->wdt, base + i);
        a->y[(size_t)r * a->out + o] = v;
    }
}

/* y[r, o] = sum_i x[r, i] * W[o, i]   (Linear::Forward, Mac/cpu/src/linear.cpp:69-81; no bias in Qwen3). */
void oracle_linear(const float* x, int rows, int in, const void* w, int wdt, int out, float* y) {
    lin_ctx c = {x, in, wdt, out, w, y};
    par_for((long)rows * out, in, lin_range, &c);
}

/* RMSNorm over the last dim (RMSNormModule::Forward, Mac/cpu/src/rms_norm_module.cpp:52-66). */
void oracle_rmsnorm(const float* x, int rows, int n, const void* w, int wdt, float eps, float* y) {
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * n;
        float* yr = y + (size_t)r * n;
        float ms = 0.0f;
        for (int i = 0; i < n; ++i) ms += xr[i] * xr[i];
        ms /= (float)n;
        const float s = 1.0f / sqrtf(ms + eps);
        for (int i = 0; i < n; ++i) yr[i] = xr[i] * s * rd(w, wdt, i);
    }
}

/* Rotate-half RoPE in place on [T, heads, D] at absolute positions pos0 + t
 * (RoPE::ApplyInPlace, Mac/cpu/src/rope.cpp:54-89: angle in double, cos/sin cast to float). */
void oracle_rope(float* x, int T, int heads, int D, double theta, int pos0) {
    const int half = D / 2;
    for (int t = 0; t < T; ++t) {
        const double ap = (double)(pos0 + t);
        for (int h = 0; h < heads; ++h) {
            float* hb = x + ((size_t)t * heads + h) * D;
            for (int i = 0; i < half; ++i) {
                const double ex = (double)(i * 2) / (double)D;
                const double ang = ap / pow(theta, ex);
                const float c = (float)cos(ang);
                const float s = (float)sin(ang);
                const float a = hb[i], b = hb[i + half];
                hb[i] = a * c - b * s;
                hb[i + half] = a * s + b * c;
            }
        }
    }
}

typedef struct {
    const float *q, *k, *v;
    float* out;
    int Hq, S, Hkv, D, prefix;
} att_ctx;

static void att_range(void* c, long lo, long hi) {
    const att_ctx* a = (const att_ctx*)c;
    const int Hq = a->Hq, Hkv = a->Hkv, D = a->D, S = a->S;
    const int group = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)D);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    float* wts = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    for (long j = lo; j < hi; ++j) {
        const int t = (int)(j / Hq), h = (int)(j % Hq);
        int vis = a->prefix + t + 1;
        if (vis > S) vis = S;
        const int kh = h / group;
        const float* qv = a->q + ((size_t)t * Hq + h) * D;
        float mx = -INFINITY;
        for (int p = 0; p < vis; ++p) {
            const float* kv = a->k + ((size_t)p * Hkv + kh) * D;
            float sc = 0.0f;
            for (int d = 0; d < D; ++d) sc += qv[d] * kv[d];
            sc *= scale;
            scores[p] = sc;
            if (sc > mx) mx = sc;
        }
        float sum = 0.0f;
        for (int p = 0; p < vis; ++p) {
            const float wv = expf(scores[p] - mx);
            wts[p] = wv;
            sum += wv;
        }
        float* o = a->out + ((size_t)t * Hq + h) * D;
        for (int d = 0; d < D; ++d) o[d] = 0.0f;
        for (int p = 0; p < vis; ++p) {
            const float nw = wts[p] / sum;
            const float* vv = a->v + ((size_t)p * Hkv + kh) * D;
            for (int d = 0; d < D; ++d) o[d] += nw * vv[d];
        }
    }
    free(scores);
    free(wts);
}

/* Causal GQA with a cached prefix (GroupedQueryAttention::ForwardWithPrefix,
 * Mac/cpu/src/grouped_query_attention.cpp:59-142).
 * q [T, Hq, D]; k, v [S, Hkv, D]; out [T, Hq, D]. */
void oracle_attention(const float* q, int T, int Hq, const float* k, const float* v, int S, int Hkv, int D,
                      int prefix, float* out) {
    att_ctx c = {q, k, v, out, Hq, S, Hkv, D, prefix};
    par_for((long)T * Hq, (long)(prefix + T) * D * 2, att_range, &c);
}

/* Greedy pick: first strict maximum (Sampler::SampleFromLogits with top_k = 1,
 * Mac/cpu/src/sampler.cpp:26-62 -- partial_sort keeps the lowest index on ties). */
int oracle_argmax(const float* logits, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* ---- whole model ---------------------------------------------------------
 * Layer tensor slots, in the order of soc_b200.bundle.layer_tensor_names. */
enum {
    W_IN_NORM = 0, W_Q, W_K, W_V, W_O, W_Q_NORM, W_K_NORM, W_POST_NORM, W_GATE, W_UP, W_DOWN, W_PER_LAYER
};

typedef struct {
    int hidden, inter, layers, hq, hkv, hd, vocab, max_seq;
    float eps;
    double theta;
    const void* embed;   int embed_dt;
    const void* fnorm;   int fnorm_dt;
    const void* lm_head; int lm_head_dt; /* NULL when tied to embed */
    const void** lw;     const int* lw_dt; /* layers * W_PER_LAYER */
    float* kcache;       /* [L][Hkv][max_seq][D] fp32, like TensorKVCache (kv_cache.cpp:148-155) */
    float* vcache;
    int length;          /* cached positions */
} oracle_model;

static inline size_t kv_off(const oracle_model* m, int l, int h, int p) {
    return (((size_t)l * m->hkv + h) * m->max_seq + p) * m->hd;
}

/* ForwardLogitsCached (Mac/cpu/src/qwen_causal_lm.cpp:58-64,74-80,82-116) for batch 1:
 * embed -> L x QwenBlock::ForwardCached (qwen_block.cpp:63-72) -> final norm -> logits of
 * the rows [first_row, T).  Returns 0, or -1 for an out-of-range id (embedding.cpp:66-68),
 * -2 for a cache overflow (kv_cache.cpp:50-52). */
int oracle_forward_cached(oracle_model* m, const int32_t* ids, int T, int pos, float* logits, int first_row) {
    const int H = m->hidden, I = m->inter, D = m->hd, Hq = m->hq, Hkv = m->hkv;
    const int QN = Hq * D, KN = Hkv * D;
    if (pos + T > m->max_seq) return -2;
    for (int t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= m->vocab) return -1;
    float* h = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* xn = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)T * QN);
    float* k = (float*)malloc(sizeof(float) * (size_t)T * KN);
    float* v = (float*)malloc(sizeof(float) * (size_t)T * KN);
    float* qn = (float*)malloc(sizeof(float) * (size_t)T * QN);
    float* kn = (float*)malloc(sizeof(float) * (size_t)T * KN);
    float* att = (float*)malloc(sizeof(float) * (size_t)T * QN);
    float* ao = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* g = (float*)malloc(sizeof(float) * (size_t)T * I);
    float* u = (float*)malloc(sizeof(float) * (size_t)T * I);
    const int S = pos + T;
    float* kall = (float*)malloc(sizeof(float) * (size_t)S * KN);
    float* vall = (float*)malloc(sizeof(float) * (size_t)S * KN);

    for (int t = 0; t < T; ++t)
        for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = rd(m->embed, m->embed_dt, (size_t)ids[t] * H + i);

    for (int l = 0; l < m->layers; ++l) {
        const void* const* w = m->lw + (size_t)l * W_PER_LAYER;
        const int* dt = m->lw_dt + (size_t)l * W_PER_LAYER;
        oracle_rmsnorm(h, T, H, w[W_IN_NORM], dt[W_IN_NORM], m->eps, xn);
        oracle_linear(xn, T, H, w[W_Q], dt[W_Q], QN, q);
        oracle_linear(xn, T, H, w[W_K], dt[W_K], KN, k);
        oracle_linear(xn, T, H, w[W_V], dt[W_V], KN, v);
        /* qwen_attention.cpp:168-171: per-head q/k norm then RoPE at pos + t */
        oracle_rmsnorm(q, T * Hq, D, w[W_Q_NORM], dt[W_Q_NORM], m->eps, qn);
        oracle_rmsnorm(k, T * Hkv, D, w[W_K_NORM], dt[W_K_NORM], m->eps, kn);
        oracle_rope(qn, T, Hq, D, m->theta, pos);
        oracle_rope(kn, T, Hkv, D, m->theta, pos);
        /* qwen_attention.cpp:180-193: TensorKVCache::Write of post-RoPE K and raw V */
        for (int t = 0; t < T; ++t)
            for (int hh = 0; hh < Hkv; ++hh)
                for (int d = 0; d < D; ++d) {
                    m->kcache[kv_off(m, l, hh, pos + t) + d] = kn[((size_t)t * Hkv + hh) * D + d];
                    m->vcache[kv_off(m, l, hh, pos + t) + d] = v[((size_t)t * Hkv + hh) * D + d];
                }
        /* qwen_attention.cpp:196-197: rebuild [S, Hkv, D] from the cache */
        for (int p = 0; p < S; ++p)
            for (int hh = 0; hh < Hkv; ++hh)
                for (int d = 0; d < D; ++d) {
                    kall[((size_t)p * Hkv + hh) * D + d] = m->kcache[kv_off(m, l, hh, p) + d];
                    vall[((size_t)p * Hkv + hh) * D + d] = m->vcache[kv_off(m, l, hh, p) + d];
                }
        oracle_attention(qn, T, Hq, kall, vall, S, Hkv, D, pos, att);
        oracle_linear(att, T, QN, w[W_O], dt[W_O], H, ao);
        for (size_t i = 0; i < (size_t)T * H; ++i) h[i] = h[i] + ao[i];      /* AddTensors */
        oracle_rmsnorm(h, T, H, w[W_POST_NORM], dt[W_POST_NORM], m->eps, xn);
        oracle_linear(xn, T, H, w[W_GATE], dt[W_GATE], I, g);
        oracle_linear(xn, T, H, w[W_UP], dt[W_UP], I, u);
        for (size_t i = 0; i < (size_t)T * I; ++i) {                         /* qwen_mlp.cpp:20-54 */
            const float a = g[i] / (1.0f + expf(-g[i]));
            g[i] = a * u[i];
        }
        oracle_linear(g, T, I, w[W_DOWN], dt[W_DOWN], H, ao);
        for (size_t i = 0; i < (size_t)T * H; ++i) h[i] = h[i] + ao[i];
    }
    oracle_rmsnorm(h, T, H, m->fnorm, m->fnorm_dt, m->eps, xn);
    if (logits != NULL && first_row < T) {
        const void* lw = m->lm_head ? m->lm_head : m->embed;
        const int ldt = m->lm_head ? m->lm_head_dt : m->embed_dt;
        oracle_linear(xn + (size_t)first_row * H, T - first_row, H, lw, ldt, m->vocab, logits);
    }
    if (pos + T > m->length) m->length = pos + T;
    free(h); free(xn); free(q); free(k); free(v); free(qn); free(kn); free(att); free(ao);
    free(g); free(u); free(kall); free(vall);
    return 0;
}
