/*
 * guanaco_b200.h -- C ABI of libguanaco_b200.so, the sm_100a (B200) decode
 * hot path for the Guanaco GGUF inference engine.
 *
 * Two layers of entry points:
 *
 *  1. DROP-IN SYMBOLS.  Exactly the extern "C" functions the unchanged Guanaco
 *     engine, loader and KV cache bind when built with USE_CUDA=1; linking this
 *     library in place of the reference CUDA sources (src/kernels/cuda) and src/backend/cuda_backend.c
 *     replaces the reference CUDA path.  Each declaration cites the reference
 *     interface it replaces (paths relative to the Guanaco repo root).  The
 *     vtable factory (backend_cuda_create / backend_cuda_destroy) is declared in
 *     guanaco_backend_abi.h because it needs the reference's struct types.
 *
 *  2. NATIVE API (gb_*).  Device-pointer kernels and a device-resident decode
 *     model used by the drop-in symbols, the tests and the benchmark.  All
 *     pointers are device pointers unless the parameter name starts with h_;
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *
 * Return codes: 0 success; -1 NULL/bad dtype/ndim; -2 cols not a multiple of
 * the block width; -3 byte_size too small (these three follow
 * src/kernels/cpu/quant_matvec_q4_k.c:143-158); -4 position outside
 * [0, max_seq); -5 CUDA runtime error; -6 out of device memory; -7 a bounded
 * device wait ran out; -8 size above a documented maximum.
 *
 * dtype codes follow the reference DataType enum (src/include/types.h:16-24):
 * F32 = 0, F16 = 1, Q8_0 = 2, Q4_K = 4, Q6_K = 5; Q5_K, which that enum lacks
 * (the reference loader sizes it, src/engine/loader.c:98,117, and rejects
 * it, :586-651), is 13, GGML's type number.  F16 rows are handled in
 * "blocks" of 32 halves (64 bytes).  gb_matvec / gb_matvec_host / gb_gemm /
 * gb_dequant / gb_model_set_matrix / the output head take Q5_K and F16 too;
 * the reference-facing vtable slots and layer ABI keep the reference's set.
 */
#ifndef GUANACO_B200_H
#define GUANACO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ========================================================================
 * 1. Drop-in symbols
 * ===================================================================== */

/* Replaces cuda_upload_weight (src/kernels/cuda/matvec_q4k_cuda.cu:115-133,
 * called by src/engine/loader.c:713): copy `size` bytes of GGUF blocks to the
 * device; returns the device pointer or NULL (the loader then keeps the tensor
 * on the CPU).  Safe to call on mmap'd MAP_PRIVATE pages. */
void* cuda_upload_weight(const void* host_ptr, size_t size);

/* Replaces cuda_matvec_q4k_f32_impl (src/kernels/cuda/matvec_q4k_cuda.cu:85-113,
 * used by src/backend/cuda_backend.c:35-40 and tests/test_quant.c:245-281):
 * y = W x for a device-resident Q4_K matrix, host x and y, synchronous. */
int cuda_matvec_q4k_f32_impl(const void* W_data, const float* x, float* y, int num_rows, int num_cols);

/* Replaces cuda_transformer_layer_gpu (src/kernels/cuda/cuda_layer_kernels.cu:605-713,
 * declared src/include/kernels.h:46-58, called src/engine/engine.c:334-346):
 * one full decode layer (T = 1) with device-resident Q4_K / Q6_K / Q8_0
 * weights.  h_hidden is host in/out; h_k_cache / h_v_cache are the layer's
 * host KV bases ([n_kv][max_seq][head_dim] fp32, head_stride = max_seq*hd);
 * the appended K/V row is also written back into them.  Asynchronous: the
 * caller syncs with cuda_finish_layer() before reading h_hidden.  Non-zero
 * return makes the engine run the CPU layer instead (engine.c:347-349). */
int cuda_transformer_layer_gpu(
    const void* wq, int wq_rows, int wq_cols, int wq_dtype,
    const void* wk, int wk_rows, int wk_cols, int wk_dtype,
    const void* wv, int wv_rows, int wv_cols, int wv_dtype,
    const void* wo, int wo_rows, int wo_cols, int wo_dtype,
    const void* w_gate, int gate_rows, int gate_cols, int gate_dtype,
    const void* w_up, int up_rows, int up_cols, int up_dtype,
    const void* w_down, int down_rows, int down_cols, int down_dtype,
    const float* h_rms_att, const float* h_rms_ffn,
    float* h_hidden,
    float* h_k_cache, float* h_v_cache, int head_stride,
    int H, int n_heads, int n_kv_heads, int head_dim,
    int pos, int layer, int max_seq_len);

/* Replaces cuda_finish_layer (src/kernels/cuda/cuda_layer_kernels.cu:715-717,
 * called src/engine/engine.c:321): wait for all queued layer work. */
void cuda_finish_layer(void);

/* Replaces cuda_sync_kv_cache (src/kernels/cuda/cuda_layer_kernels.cu:585-603,
 * called src/engine/engine.c:398-403): upload positions [pos, pos+T) of one
 * layer's host KV into the device cache after a CPU prefill. */
void cuda_sync_kv_cache(int layer, int n_kv_heads, int head_dim, int pos, int T,
                        const float* h_k_cache, const float* h_v_cache, int stride0, int max_seq);

/* Replaces cuda_get_temperature (src/backend/cuda_backend.c:26-33, called
 * src/engine/generate.c:284): GPU temperature in C, 0 when unknown. */
int cuda_get_temperature(void);

/* ========================================================================
 * 2. Native API
 * ===================================================================== */

/* Library / device information. */
const char* gb_version(void);
int gb_device_sm_count(void);

/* y[rows] = W[rows, cols] . x[cols] (+ residual[rows] when residual != NULL).
 * W: GGUF blocks, 16-byte aligned (row tiles are fetched with bulk copies);
 * x: 16-byte aligned.  y may alias residual.  The kernel's bounded waits
 * report through gb_device_error().  Launched with programmatic dependent
 * launch: right after another matvec of this library on the same stream it
 * starts fetching W before that one has finished (x, residual and y are
 * touched only after it), so W must not be written by the kernel just before
 * it on the stream unless that kernel runs to completion first (any kernel
 * that does not execute griddepcontrol.launch_dependents does). */
int gb_matvec(int dtype, const void* W, int rows, int cols, const float* x, float* y,
              const float* residual, void* stream);

/* y_i = W_i . x for n <= 3 matrices that share x (all with cols columns):
 * one launch with one work split when the formats allow it (the decode
 * step's q/k/v and gate/up launches), else one launch per matrix.  The same
 * alignment rules as gb_matvec.  No counterpart in the reference, which
 * runs one matvec per weight (src/engine/engine.c:362-371, 533-543). */
int gb_matvec_group(int n, const int* dtypes, const void* const* W, const int* rows, int cols, const float* x,
                    float* const* y, void* stream);

/* Sticky device error word set by the library's kernels (0 = none, -7 for a
 * bounded wait that ran out).  Synchronous; clear != 0 resets it. */
int gb_device_error(int clear);

/* The same product with host x[cols] / y[rows] (copies in, sync out): the path
 * behind the backend vtable's matvec slots. */
int gb_matvec_host(int dtype, const void* W, int rows, int cols, const float* h_x, float* h_y);

/* Bit-exact dequantisation of nblocks GGUF blocks into fp32 (256 values per
 * Q4_K / Q6_K / Q5_K block, 32 per Q8_0 block or F16 block of 32 halves). */
int gb_dequant(int dtype, const void* blocks, size_t nblocks, float* out, void* stream);

/* Seeded synthetic inputs, byte-identical to the CPU generators in the test
 * oracle: blocks with the value distributions of the benchmark configs and
 * approximately N(0,1) floats (sum of twelve uniforms). */
int gb_synth_blocks(int dtype, void* blocks, size_t nblocks, uint64_t seed, uint64_t stream_id, void* stream);
int gb_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream_id, void* stream);
int gb_fill_f32(float* out, size_t n, float value, void* stream);

/* RoPE table for positions [0, max_seq): cs[(pos*head_dim/2 + i)*2 + {0,1}] =
 * {cos, sin}(pos * freq_i), freq_i = 1/theta^(2i/head_dim), computed on the
 * host with the reference's float formula (src/kernels/cpu/kernels_cpu.c:408-413)
 * and uploaded.  cs holds max_seq * head_dim floats. */
int gb_rope_table(float* cs, int max_seq, int head_dim, float theta, void* stream);

/* Decode attention for one layer at one position, fused with RoPE and the KV
 * append (engine.c:372-509 semantics):
 *   q[n_heads*hd] and k[n_kv*hd] are rotated (RoPE row pos of rope_cs),
 *   k_rot and v are written to slot pos of k_cache / v_cache
 *   ([n_kv][max_seq][hd] fp32), then out[n_heads*hd] = softmax(q k^T / sqrt(hd)) V
 *   over positions [0, pos].
 * pos is read from device memory (d_pos) so the call can be captured in a
 * CUDA graph.  The context is split across CTAs (split-K) and merged with an
 * online-softmax reduction in the last CTA of each KV head.
 * ws: workspace of gb_attn_workspace_bytes(...) bytes, zeroed once before the
 * first call (the kernel leaves its counters at zero on return).
 * head_dim must be 64 or 128 and n_heads/n_kv in {1, 2, 4, 8}. */
size_t gb_attn_workspace_bytes(int n_heads, int n_kv, int head_dim, int max_seq);
int gb_attention_decode(const float* q, const float* k, const float* v,
                        float* k_cache, float* v_cache, const float* rope_cs,
                        const int* d_pos, int n_heads, int n_kv, int head_dim, int max_seq,
                        float* out, void* ws, void* stream);

/* Prefill GEMM for T tokens at once on the tcgen05 tensor cores:
 * Y[t][n] = sum_k X[t][k] W[n][k] (+ R[t][n] when R is not NULL; R may be Y),
 * all device pointers, X / Y / R row-major fp32 (T x K, T x N).  W is N rows of
 * GGUF blocks (dtype 4 Q4_K, 5 Q6_K, 2 Q8_0, 13 Q5_K) or fp32 / fp16 rows
 * (dtype 0 / 1).  fp32-equivalent: weights and activations are split into
 * an 11-bit part and a remainder (hi.hi + hi.lo + lo.hi), as fp16 pairs with
 * power-of-two row scales (default) or tf32 pairs (GB_GEMM_KIND=tf32).  In
 * the fp16 form X is first split into stream-ordered scratch
 * (cudaMallocAsync, gb_gemm_split_bytes x 2 + 4 T bytes).  Replaces the
 * per-token loop of linear_dispatch (src/engine/engine.c:119-153) for T > 1;
 * the reference's GPU prefill hook is a stub (src/engine/gpu_prefill.c:3-20).
 * Asynchronous on `stream`. */
int gb_gemm(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T, void* stream);
/* The fp16 form in two steps, so that one split X serves several GEMMs (no
 * reference counterpart; the reference has no batched GEMM): gb_gemm_split
 * writes hi and lo (gb_gemm_split_bytes(T, K) bytes each, 16-byte aligned)
 * and inv (T floats); gb_gemm_presplit then computes Y as gb_gemm does from
 * a split made with the same T and K (the layout's row pitch is T rounded up
 * to 256).  K a multiple of 32.  GB_EINVAL when GB_GEMM_KIND=tf32. */
size_t gb_gemm_split_bytes(int T, int K);
int gb_gemm_split(const float* X, int T, int K, void* hi, void* lo, float* inv, void* stream);
int gb_gemm_presplit(int dtype, const void* W, const void* hi, const void* lo, const float* inv, float* Y,
                     const float* R, int N, int K, int T, void* stream);
/* Device error word of the GEMM's bounded waits (GB_ETIMEOUT); clear != 0
 * resets it. */
int gb_gemm_error(int clear);

/* Causal attention of a prompt's n_tokens query rows (positions pos ..
 * pos + n_tokens - 1) over the device KV cache of one layer, whose rows
 * [0, pos + n_tokens) are filled: out[t][h*hd..] = softmax over keys
 * s <= pos + t of (q_t . k_s) / sqrt(hd), times v_s.  q / out row-major
 * [n_tokens][n_heads * head_dim]; caches [n_kv][max_seq][hd].  The T > 1
 * attention of transformer_layer (src/engine/engine.c:431-500), on the tensor
 * cores (fp32-equivalent 3xTF32 scores and P.V, fp32 softmax).  head_dim 64
 * or 128; n_heads / n_kv_heads in {1, 2, 4, 8}.  Asynchronous on `stream`. */
int gb_prefill_attention(const float* q, const float* k_cache, const float* v_cache, float* out, int n_tokens,
                         int pos, int n_heads, int n_kv_heads, int head_dim, int max_seq, void* stream);
/* Device error word of gb_prefill_attention's bounded waits (GB_ETIMEOUT);
 * clear != 0 resets it. */
int gb_prefill_attention_error(int clear);

/* Frees every device copy the vtable matvec slots made of weights that were
 * never uploaded (the engine's lm_head).  Those copies are keyed by host
 * pointer and checked against the byte size and a checksum of sampled
 * bytes; a caller that edits a weight in place after its first use calls
 * this before the next matvec.  The cache also drops its least recently used
 * copies above GB_VTABLE_CACHE_MB (environment, default 16384 MiB).
 * Synchronises the library's stream.  No counterpart in the reference, whose
 * CUDA backend fell back to the CPU for such tensors. */
int gb_vtable_cache_clear(void);

/* gb_attention_decode without a caller workspace and without allocating:
 * the split-K scratch is a file-scope device array of GB_ATTN_STATIC_BYTES
 * (4 MiB), resolved with cudaGetSymbolAddress once per device.  Returns
 * GB_ELIMIT when the configuration needs more (partials of n_kv * splits *
 * (n_heads / n_kv) * (head_dim + 4) floats above 4 MiB - 4 KiB, or n_kv >= 1023).
 * The scratch is shared by every call on the device: calls that overlap in
 * time (other streams, other threads) race and must not be issued.  The first
 * call on a device does the symbol lookup, so make it before any stream
 * capture.  The looked-up address belongs to the device's primary context: a
 * process that calls cudaDeviceReset on a device must not call this entry
 * point on that device afterwards.  A position outside [0, max_seq) is
 * reported through gb_attention_static_error (after synchronising the stream). */
#define GB_ATTN_STATIC_BYTES (4u << 20)
int gb_attention_decode_static(const float* q, const float* k, const float* v,
                               float* k_cache, float* v_cache, const float* rope_cs,
                               const int* d_pos, int n_heads, int n_kv, int head_dim, int max_seq,
                               float* out, void* stream);
/* The static variant's error word as a GB_E* code (0 if none); clear != 0
 * resets it. */
int gb_attention_static_error(int clear);

/* out = w * (x * rsqrt(mean(x^2) + eps))  (kernels_cpu.c:199-265), one row of n. */
int gb_rmsnorm(const float* x, const float* w, float* out, int n, float eps, void* stream);
/* gate = silu(gate) * up  (kernels_cpu.c:312-341 + 367-389). */
int gb_silu_mul(float* gate, const float* up, int n, void* stream);
/* first index of the maximum (strict >, src/tokenizer/tokenizer.c:175-185). */
int gb_argmax(const float* x, int n, int* d_out, void* stream);

/* ---- Device-resident decode model (the fast path behind forward()) ---- */
typedef struct gb_model gb_model;

typedef struct {
    int hidden_dim, n_heads, n_kv_heads, head_dim, n_layers, ff_dim, vocab_size, max_seq;
    float rms_eps;      /* the reference hard-codes 1e-6 (engine.c:359,524,582) */
    float rope_theta;   /* the reference hard-codes 500000 (kernels_cpu.c:408) */
} gb_model_config;

/* Matrix slots per layer, in this order. */
enum { GB_WQ = 0, GB_WK, GB_WV, GB_WO, GB_WGATE, GB_WUP, GB_WDOWN, GB_NMAT };

/* Allocate activations, KV cache, RoPE table and workspaces on the current
 * device.  Weights are attached separately. */
/* Tensor-parallel slice `rank` of `world` (1..8) GPUs, one process per GPU:
 * q / k / v rows and wo columns of this rank's n_heads / world query heads and
 * n_kv_heads / world KV heads (attention and its KV cache stay local), gate /
 * up rows and ffn_down columns of its ff_dim / world FFN slice, output-head
 * rows [vocab_off, vocab_off + vocab_rows).  After wo and ffn_down the ranks'
 * partial hidden vectors are summed over NVLink peer memory (in rank order:
 * every rank holds the same hidden state); the greedy token is the best of the
 * ranks' slices.  A Q6_K ffn_down shard is stored with its rows padded to a
 * multiple of 8 blocks (zero blocks after the shard's columns).  Requires
 * n_kv_heads % world == 0, ff_dim % (256 * world) == 0 and
 * (n_heads / world * head_dim) % 256 == 0.  Before decoding, exchange the
 * ranks' handles: gb_model_comm_handle on every rank, then gb_model_comm_open
 * with all world handles (GB_IPC_HANDLE_BYTES each, in rank order).  Every
 * rank must run the same sequence of decode calls (the exchanges pair them). */
gb_model* gb_model_create_tp(const gb_model_config* cfg, int rank, int world);
#define GB_IPC_HANDLE_BYTES 64
int gb_model_comm_handle(gb_model* m, void* handle);
int gb_model_comm_open(gb_model* m, const void* handles);
int gb_model_tp_info(const gb_model* m, int* rank, int* world, int* vocab_off, int* vocab_rows);
gb_model* gb_model_create(const gb_model_config* cfg);
void gb_model_destroy(gb_model* m);

/* Attach weights by device pointer (the model does not own them).
 * which = GB_WQ..GB_WDOWN; norms are fp32 [hidden_dim]. */
int gb_model_set_matrix(gb_model* m, int layer, int which, int dtype, const void* d_w);
int gb_model_set_norms(gb_model* m, int layer, const float* d_rms_att, const float* d_rms_ffn);
int gb_model_set_head(gb_model* m, int emb_dtype, const void* d_embedding, const float* d_rms_final,
                      int lm_dtype, const void* d_lm_head);

/* Allocate and fill every weight with seeded synthetic blocks (Q4_K_M-style
 * mix: Q4_K everywhere except Q6_K for wv, w_down and lm_head; norms 1.0;
 * Q4_K embedding).  The model owns these buffers. */
int gb_model_synthesize(gb_model* m, uint64_t seed);

/* Device KV cache of one layer ([n_kv][max_seq][hd] fp32 each). */
float* gb_model_k_cache(gb_model* m, int layer);
float* gb_model_v_cache(gb_model* m, int layer);

/* One decode step for token at position pos (forward() of engine.c:559-594
 * at T = 1, then greedy argmax).  Everything stays on the device:
 * d_logits (may be NULL) receives vocab_size logits, d_next the argmax.
 * The step is captured once into a CUDA graph and replayed. */
int gb_model_decode(gb_model* m, const int* d_token, const int* d_pos, float* d_logits, int* d_next,
                    void* stream);

/* Same step with host token/position in and host next token (and optionally
 * host logits) out: the end-to-end entry point. */
int gb_model_decode_host(gb_model* m, int token, int pos, int* h_next, float* h_logits);
/* (h_logits / d_logits receive this rank's vocabulary rows; all of them on one GPU.) */

/* Prefill: forward() of engine.c:559-594 for a prompt of n_tokens tokens at
 * positions pos .. pos + n_tokens - 1 -- what the reference's GPU prefill
 * hook gpu_prefill(backend, model, kv, scr, token_ids, n_tokens, pos)
 * (src/engine/gpu_prefill.c:3-20, a stub there) is for.  Every layer runs
 * over all the prompt's rows at once (tensor-core GEMMs, causal attention),
 * the K / V cache rows pos .. pos + n_tokens - 1 are written, and the last
 * row's logits (d_logits, may be NULL) and argmax (d_next) come out, so
 * decode continues at pos + n_tokens.  Long prompts run in chunks of 4096
 * rows (GB_PREFILL_CHUNK).  One GPU (world 1).  Asynchronous on `stream`;
 * returns GB_EPOS when pos + n_tokens > max_seq.  Activation buffers are
 * allocated by the first call and kept with the model. */
int gb_model_prefill(gb_model* m, const int* d_tokens, int n_tokens, int pos, float* d_logits, int* d_next,
                     void* stream);
/* Same with the prompt on the host and the next token (and optionally the
 * logits) returned to the host; synchronous. */
int gb_model_prefill_host(gb_model* m, const int* h_tokens, int n_tokens, int pos, int* h_next, float* h_logits);

/* Greedy generation entirely on the device: n_steps replays of a graph that
 * runs one decode step and then feeds the argmax back (*d_token = next,
 * *d_pos += 1).  Step i's token goes to d_tokens_out[i] when not NULL.
 * Asynchronous on `stream`. */
int gb_model_generate(gb_model* m, int* d_token, int* d_pos, int n_steps, int* d_tokens_out, void* stream);

/* Fill positions [0, n_pos) of every layer's K and V cache with seeded
 * synthetic values (approximately N(0,1)): a stand-in for a prefilled context. */
int gb_model_fill_kv(gb_model* m, int n_pos, uint64_t seed);

/* Device error word of the model (0 = none; e.g. -4 for a position outside
 * [0, max_seq) or -1 for a token outside the vocabulary).  Synchronises. */
int gb_model_error(gb_model* m);

/* Kernel launches one decode step issues. */
int gb_model_launches_per_step(const gb_model* m);

/* Byte count of one decode step's algorithmic HBM traffic at position pos
 * (weights + KV read + KV append + activations), for rooflines. */
double gb_model_step_bytes(const gb_model* m, int pos);

#ifdef __cplusplus
}
#endif
#endif /* GUANACO_B200_H */
