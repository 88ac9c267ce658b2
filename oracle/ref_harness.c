/*
 * ref_harness.c -- thin C entry points over the UNMODIFIED Guanaco reference
 * CPU code, compiled from the reference tree where it lies (oracle/Makefile)
 * into oracle/_ref/libref.so.  TEST INFRASTRUCTURE ONLY: it pins the oracle
 * restatement (gb_oracle.c) and is the CPU baseline that bench.py times.
 *
 * engine.c is included textually so that its file-static embedding_lookup
 * (the only standalone dequantiser in the reference, engine.c:214-283) can be
 * reached; nothing in it is changed.
 */
#include "engine.c"   /* src/engine/engine.c, unmodified */

#include "backend.h"
#include "kernels_ext.h"
#include "quant.h"
#include "threadpool.h"

#include <stdlib.h>
#include <string.h>

extern void kernels_cpu_set_threadpool(ThreadPool* tp);

static ThreadPool* g_ref_pool = NULL;

/* Use n host threads in the reference kernels that fan out (Q4_K matvec,
 * gemm_f32, gemm_f32_nn); Q6_K and Q8_0 are single-threaded by construction. */
void ref_set_threads(int n) {
    if (g_ref_pool) {
        kernels_cpu_set_threadpool(NULL);
        threadpool_destroy(g_ref_pool);
        g_ref_pool = NULL;
    }
    if (n > 1) {
        g_ref_pool = threadpool_create(n);
        kernels_cpu_set_threadpool(g_ref_pool);
    }
}

static Tensor make_q_tensor(int dtype, const void* W, int rows, int cols, size_t byte_size) {
    Tensor t;
    memset(&t, 0, sizeof(t));
    t.data = (void*)W;
    t.ndim = 2;
    t.shape[0] = rows;
    t.shape[1] = cols;
    t.stride[0] = cols;
    t.stride[1] = 1;
    t.dtype = (DataType)dtype;
    t.byte_size = byte_size;
    return t;
}

/* The three vtable matvec slots (quant_matvec_q4_k.c:142, _q6_k.c:43, _q8_0.c:41). */
int ref_matvec(int dtype, const void* W, int rows, int cols, size_t byte_size,
               const float* x, float* y) {
    Tensor t = make_q_tensor(dtype, W, rows, cols, byte_size);
    switch (dtype) {
        case DTYPE_Q4_K: return matvec_q4k_f32(&t, x, y);
        case DTYPE_Q6_K: return matvec_q6k_f32(&t, x, y);
        case DTYPE_Q8_0: return matvec_q8_0_f32(&t, x, y);
        default: return -1;
    }
}

/* Dequantise nblocks of Q4_K (dtype 4) or nblocks of Q8_0 (dtype 2) through
 * embedding_lookup on a one-row embedding table. */
int ref_dequant(int dtype, const void* blocks, int nblocks, float* out) {
    const int per = dtype == DTYPE_Q4_K ? 256 : 32;
    Tensor emb = make_q_tensor(dtype, blocks, 1, nblocks * per, 0);
    Tensor o;
    memset(&o, 0, sizeof(o));
    o.data = out;
    o.ndim = 2;
    o.shape[0] = 1;
    o.shape[1] = nblocks * per;
    o.dtype = DTYPE_F32;
    int tok = 0;
    if (dtype != DTYPE_Q4_K && dtype != DTYPE_Q8_0) return -1;
    embedding_lookup(&emb, &tok, 1, &o);
    return 0;
}

static KernelVTable ref_vtable(void) {
    KernelVTable k;
    memset(&k, 0, sizeof(k));
    k.gemm_f32 = gemm_f32;
    k.gemm_f32_nn = gemm_f32_nn;
    k.rmsnorm = cpu_rmsnorm;
    k.softmax_inplace = softmax_inplace;
    k.silu_inplace = silu_inplace;
    k.rope = rope;
    k.residual_add = residual_add;
    k.elemwise_mul = elemwise_mul;
    k.matvec_q4k_f32 = matvec_q4k_f32;
    k.matvec_q6k_f32 = matvec_q6k_f32;
    k.matvec_q8_0_f32 = matvec_q8_0_f32;
    return k;
}

/* RoPE + kv_cache_append + the attention block of transformer_layer for one
 * layer at T = 1, composed from the reference kernels exactly as
 * engine.c:372-509 composes them.  q (n_heads*hd) and k, v (n_kv*hd) are the
 * pre-RoPE projections; k_cache / v_cache are the caller's head-major
 * [n_kv][max_seq][hd] arrays (in/out; the appended row is written back);
 * q and k are rotated in place; out is (n_heads*hd). */
int ref_attention_step(float* q, float* k, const float* v, float* k_cache, float* v_cache,
                       int n_heads, int n_kv, int hd, int max_seq, int pos, float* out) {
    ModelConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.hidden_dim = n_heads * hd;
    cfg.n_heads = n_heads;
    cfg.n_kv_heads = n_kv;
    cfg.head_dim = hd;
    cfg.n_layers = 1;
    cfg.max_seq_len = max_seq;
    const size_t cache_bytes = (size_t)n_kv * max_seq * hd * sizeof(float);
    Arena* arena = arena_create(2 * cache_bytes + (1 << 20));
    if (!arena) return -2;
    KVCache* kv = kv_cache_create(arena, &cfg, max_seq);
    if (!kv) { arena_destroy(arena); return -2; }
    memcpy(kv_cache_raw_k(kv, 0), k_cache, cache_bytes);
    memcpy(kv_cache_raw_v(kv, 0), v_cache, cache_bytes);

    KernelVTable kt = ref_vtable();
    Tensor qv = make_view(q, 2, n_heads, hd, 0);
    Tensor kv_t = make_view(k, 2, n_kv, hd, 0);
    kt.rope(&qv, &kv_t, pos, hd);
    Tensor vv = make_view((float*)v, 2, n_kv, hd, 0);
    kv_cache_append(kv, 0, &kv_t, &vv, pos);

    const int seq_len = pos + 1;
    Tensor* K_cached = kv_cache_get_k(kv, 0, seq_len);
    Tensor* V_cached = kv_cache_get_v(kv, 0, seq_len);
    float* scores = (float*)malloc((size_t)seq_len * sizeof(float));
    float* ctx = (float*)malloc((size_t)hd * sizeof(float));
    Tensor sc_t = make_view(scores, 2, 1, seq_len, 0);
    Tensor ctx_t = make_view(ctx, 2, 1, hd, 0);
    const float scale = 1.0f / sqrtf((float)hd);
    const int heads_per_kv = n_heads / n_kv;
    for (int h = 0; h < n_heads; h++) {
        const int kv_h = h / heads_per_kv;
        Tensor q_pack = make_view(q + (size_t)h * hd, 2, 1, hd, 0);
        float* k_h = (float*)K_cached->data + (size_t)kv_h * K_cached->stride[0];
        float* v_h = (float*)V_cached->data + (size_t)kv_h * V_cached->stride[0];
        Tensor K_head = make_view(k_h, 2, seq_len, hd, 0);
        Tensor V_head = make_view(v_h, 2, seq_len, hd, 0);
        kt.gemm_f32(&q_pack, &K_head, &sc_t);
        for (int s = 0; s < seq_len; s++) {
            float val = scores[s] * scale;
            if (s > pos) val = -INFINITY;
            scores[s] = val;
        }
        kt.softmax_inplace(&sc_t, seq_len);
        kt.gemm_f32_nn(&sc_t, &V_head, &ctx_t);
        memcpy(out + (size_t)h * hd, ctx, (size_t)hd * sizeof(float));
    }
    memcpy(k_cache, kv_cache_raw_k(kv, 0), cache_bytes);
    memcpy(v_cache, kv_cache_raw_v(kv, 0), cache_bytes);
    free(scores);
    free(ctx);
    kv_cache_destroy(kv);
    arena_destroy(arena);
    return 0;
}

/* A small model description for forward(): weights are raw block pointers in
 * the GGUF layout with reference dtype codes; norms are fp32.  Per layer the
 * seven matrices are wq, wk, wv, wo, gate, up, down. */
typedef struct {
    int H, n_heads, n_kv, hd, ff, vocab, n_layers, max_seq;
    const void* const* w;        /* n_layers * 7 pointers */
    const int* w_dtype;          /* n_layers * 7 */
    const float* const* rms_att; /* n_layers */
    const float* const* rms_ffn; /* n_layers */
    const void* embedding; int emb_dtype;
    const float* rms_final;
    const void* lm_head; int lm_dtype;
} ref_model_desc;

typedef struct {
    ModelWeights mw;
    Tensor* tensors;
    Arena* arena;
    KVCache* kv;
    Scratch* scr;
    KernelVTable kt;
    void* backend;   /* the engine's Backend (USE_CUDA build, after ref_model_to_gpu) */
    int H, kv_dim, ff, hd, vocab, n_layers, max_seq;
    int max_t;       /* prompt length the scratch holds (grown by ref_model_forward_n) */
} ref_model;

/* forward() resets the scratch once per call, so it must hold every layer's
 * temporaries (engine.c:354-546) plus the final norm and logits for a
 * prompt of T tokens; the attention scores are T x seq_len per layer. */
static size_t ref_scratch_bytes(const ref_model* m, int T) {
    const size_t per_layer = (size_t)T * (10 * m->H + 2 * m->kv_dim + 2 * m->ff + m->max_seq + 2 * m->hd) *
                                 sizeof(float) + 32 * (sizeof(Tensor) + 128);
    return (size_t)m->n_layers * per_layer + (size_t)T * (4 * m->H + 2 * m->vocab) * sizeof(float) + (1u << 20);
}

static size_t q_bytes(int dtype, int rows, int cols) {
    switch (dtype) {
        case DTYPE_Q4_K: return (size_t)rows * (cols / 256) * 144;
        case DTYPE_Q6_K: return (size_t)rows * (cols / 256) * 210;
        case DTYPE_Q8_0: return (size_t)rows * (cols / 32) * 34;
        case DTYPE_F32: return (size_t)rows * cols * 4;
        default: return 0;
    }
}

/* Build a reference ModelWeights + KVCache + Scratch over caller-owned weight
 * bytes.  Returns an opaque handle or NULL. */
void* ref_model_create(const ref_model_desc* d) {
    ref_model* m = (ref_model*)calloc(1, sizeof(ref_model));
    ModelConfig* c = &m->mw.config;
    c->hidden_dim = d->H;
    c->n_heads = d->n_heads;
    c->n_kv_heads = d->n_kv;
    c->head_dim = d->hd;
    c->n_layers = d->n_layers;
    c->vocab_size = d->vocab;
    c->ff_dim = d->ff;
    c->max_seq_len = d->max_seq;
    const int kv_dim = d->n_kv * d->hd;
    const int n_t = d->n_layers * 9 + 3;
    m->tensors = (Tensor*)calloc((size_t)n_t, sizeof(Tensor));
    m->mw.layers = (LayerWeights*)calloc((size_t)d->n_layers, sizeof(LayerWeights));
    Tensor* t = m->tensors;
    for (int l = 0; l < d->n_layers; l++) {
        const int rows[7] = {d->H, kv_dim, kv_dim, d->H, d->ff, d->ff, d->H};
        const int cols[7] = {d->H, d->H, d->H, d->H, d->H, d->H, d->ff};
        Tensor* lt[9];
        for (int i = 0; i < 7; i++) {
            const int dt = d->w_dtype[l * 7 + i];
            *t = make_q_tensor(dt, d->w[l * 7 + i], rows[i], cols[i], q_bytes(dt, rows[i], cols[i]));
            lt[i] = t++;
        }
        for (int i = 0; i < 2; i++) {
            const float* nw = i == 0 ? d->rms_att[l] : d->rms_ffn[l];
            *t = make_view((float*)nw, 1, d->H, 0, 0);
            lt[7 + i] = t++;
        }
        LayerWeights* L = &m->mw.layers[l];
        L->wq = lt[0]; L->wk = lt[1]; L->wv = lt[2]; L->wo = lt[3];
        L->w_gate = lt[4]; L->w_up = lt[5]; L->w_down = lt[6];
        L->rms_att = lt[7]; L->rms_ffn = lt[8];
    }
    *t = make_q_tensor(d->emb_dtype, d->embedding, d->vocab, d->H, q_bytes(d->emb_dtype, d->vocab, d->H));
    m->mw.embedding = t++;
    *t = make_view((float*)d->rms_final, 1, d->H, 0, 0);
    m->mw.rms_final = t++;
    *t = make_q_tensor(d->lm_dtype, d->lm_head, d->vocab, d->H, q_bytes(d->lm_dtype, d->vocab, d->H));
    m->mw.lm_head = t++;

    const size_t kv_bytes = 2 * (size_t)d->n_layers * kv_dim * d->max_seq * sizeof(float);
    m->arena = arena_create(kv_bytes + (4u << 20));
    m->kv = m->arena ? kv_cache_create(m->arena, c, d->max_seq) : NULL;
    m->H = d->H; m->kv_dim = kv_dim; m->ff = d->ff; m->hd = d->hd; m->vocab = d->vocab;
    m->n_layers = d->n_layers; m->max_seq = d->max_seq;
    m->max_t = 16;
    m->scr = scratch_create(ref_scratch_bytes(m, m->max_t));
    m->kt = ref_vtable();
    if (!m->kv || !m->scr) return NULL;
    return m;
}

/* Raw head-major K/V bases of one layer (kv_cache.c:189-205), for synthetic
 * cache fills and for comparing caches. */
float* ref_model_kv(void* h, int layer, int which_v) {
    ref_model* m = (ref_model*)h;
    return which_v ? kv_cache_raw_v(m->kv, layer) : kv_cache_raw_k(m->kv, layer);
}

/* forward() for one decode token at pos (engine.c:559-594); logits out. */
int ref_model_forward(void* h, int token, int pos, float* logits) {
    ref_model* m = (ref_model*)h;
    Tensor* lg = forward(&m->mw, m->kv, m->scr, &token, 1, pos, &m->kt);
    if (!lg) return -1;
    memcpy(logits, lg->data, (size_t)m->mw.config.vocab_size * sizeof(float));
    return 0;
}

#ifdef USE_CUDA
/* The engine's CUDA set-up (src/engine/loader.c:701-716 and
 * src/engine/generate.c:55-70), applied to the harness model: every layer
 * matrix gets a device copy through cuda_upload_weight and
 * device_residency = 1, and the kernel table comes from backend_create with
 * BACKEND_AUTO, as the engine makes it.  forward() then takes the
 * cuda_transformer_layer_gpu branch of transformer_layer (engine.c:314-350)
 * for every layer, back to back, and the output head goes through the
 * backend's matvec slot (engine.c:590).  Returns 0 when the CUDA backend was
 * selected and every layer matrix is on the device. */
extern void* cuda_upload_weight(const void* host, size_t bytes);
extern void cuda_finish_layer(void);
#include "backend_internal.h"
int ref_model_to_gpu(void* h, int threads) {
    ref_model* m = (ref_model*)h;
    int resident = 0;
    for (int l = 0; l < m->mw.config.n_layers; l++) {
        LayerWeights* L = &m->mw.layers[l];
        Tensor* ts[7] = {L->wq, L->wk, L->wv, L->wo, L->w_gate, L->w_up, L->w_down};
        for (int i = 0; i < 7; i++) {
            void* d = cuda_upload_weight(ts[i]->data, ts[i]->byte_size);
            if (d) {
                ts[i]->d_data = d;
                ts[i]->device_residency = 1;
                resident++;
            }
        }
    }
    BackendConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.kind = BACKEND_AUTO;
    cfg.threads = threads;
    cfg.device_id = 0;
    cfg.n_gpu_layers = m->mw.config.n_layers;
    Backend* b = backend_create(&cfg);
    if (!b) return -1;
    m->backend = b;
    m->kt = *backend_kernels(b);
    /* glue slots the library could not bind (it was loaded before these
     * kernels were): the engine's own CPU kernels, as the CUDA backend binds
     * them when linked into the engine */
    KernelVTable cpu = ref_vtable();
    if (!m->kt.gemm_f32) m->kt.gemm_f32 = cpu.gemm_f32;
    if (!m->kt.gemm_f32_nn) m->kt.gemm_f32_nn = cpu.gemm_f32_nn;
    if (!m->kt.rmsnorm) m->kt.rmsnorm = cpu.rmsnorm;
    if (!m->kt.softmax_inplace) m->kt.softmax_inplace = cpu.softmax_inplace;
    if (!m->kt.silu_inplace) m->kt.silu_inplace = cpu.silu_inplace;
    if (!m->kt.rope) m->kt.rope = cpu.rope;
    if (!m->kt.residual_add) m->kt.residual_add = cpu.residual_add;
    if (!m->kt.elemwise_mul) m->kt.elemwise_mul = cpu.elemwise_mul;
    return (backend_kind(b) == BACKEND_CUDA && resident == 7 * m->mw.config.n_layers) ? 0 : -2;
}
#endif

/* forward() over n prompt tokens at positions pos .. pos + n - 1 (T = n:
 * the engine's prefill, engine.c:559-594 and 353-554); logits of the last. */
int ref_model_forward_n(void* h, const int* tokens, int n, int pos, float* logits) {
    ref_model* m = (ref_model*)h;
    if (n <= 0) return -1;
    if (n > m->max_t) {   /* a longer prompt than any before: a larger scratch */
        Scratch* s2 = scratch_create(ref_scratch_bytes(m, n));
        if (!s2) return -1;
        scratch_destroy(m->scr);
        m->scr = s2;
        m->max_t = n;
    }
    int* t = (int*)malloc((size_t)n * sizeof(int));
    if (!t) return -1;
    memcpy(t, tokens, (size_t)n * sizeof(int));
    Tensor* lg = forward(&m->mw, m->kv, m->scr, t, n, pos, &m->kt);
    free(t);
    if (!lg) return -1;
    memcpy(logits, lg->data, (size_t)m->mw.config.vocab_size * sizeof(float));
    return 0;
}

void ref_model_destroy(void* h) {
    ref_model* m = (ref_model*)h;
    if (!m) return;
#ifdef USE_CUDA
    cuda_finish_layer();
    if (m->backend) backend_destroy((Backend*)m->backend);
#endif
    if (m->kv) kv_cache_destroy(m->kv);
    if (m->arena) arena_destroy(m->arena);
    if (m->scr) scratch_destroy(m->scr);
    free(m->tensors);
    free(m->mw.layers);
    free(m);
}
