/*
 * gb_oracle.h -- CPU oracle for the Guanaco decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs use it, and only as the checker.
 *
 * Every function is a plain-C11 restatement of the reference arithmetic in
 * the reference's own evaluation order (compiled with -ffp-contract=off, as
 * the reference's `-std=c11` build is), so that the results are bit-identical
 * to the reference C kernels on the same inputs.  Each function names the
 * reference file:line it restates (paths relative to the Guanaco repo root).
 *
 * Parity pin: tests/test_oracle.py checks these functions against
 *   (1) the known-answer tests of tests/test_quant.c (Q8_0 -528, Q4_K 384,
 *       Q4_K cross-byte scale/min mapping), restated as golden fixtures, and
 *   (2) the reference's own C kernels compiled unchanged into
 *       oracle/_ref/libref.so (bit-exact on seeded inputs).
 */
#ifndef GB_ORACLE_H
#define GB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- block byte sizes (loader.c:113-119) ---- */
#define GBO_Q4K_BYTES 144
#define GBO_Q6K_BYTES 210
#define GBO_Q80_BYTES 34
#define GBO_Q5K_BYTES 176   /* loader.c:117 */
#define GBO_DT_Q5_K 13      /* GGML's type number; the reference's DataType has none */

/* ---- scalar helpers ---- */
float    gbo_f16_to_f32(uint16_t h);            /* quant_matvec_q4_k.c:18-45 */
uint16_t gbo_f32_to_f16(float f);               /* IEEE round-to-nearest-even */
void     gbo_q4k_scale_min(int j, const uint8_t* q, uint8_t* d, uint8_t* m); /* :47-56 */

/* ---- dequantisation (bit-exact definitions) ---- */
void gbo_dequant_q4k(const void* blocks, size_t nblocks, float* out);  /* engine.c:248-276 */
void gbo_dequant_q6k(const void* blocks, size_t nblocks, float* out);  /* quant_matvec_q6_k.c:75-92 */
void gbo_dequant_q8_0(const void* blocks, size_t nblocks, float* out); /* engine.c:235-240 */
void gbo_dequant_q5k(const void* blocks, size_t nblocks, float* out);  /* GGML block_q5_K (no reference kernel) */
void gbo_dequant_f16(const void* blocks, size_t nblocks, float* out);  /* engine.c:183-212, blocks of 32 */

/* ---- matvec y[rows] = W[rows, cols] . x[cols]; return codes as the reference ---- */
int gbo_matvec_q4k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y);
int gbo_matvec_q6k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y);
int gbo_matvec_q8_0(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y);
int gbo_matvec_q5k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y);
int gbo_matvec_f16(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y);

/* ---- decode-layer pieces (T = 1) ---- */
void gbo_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos, float theta);
void gbo_kv_append(float* k_cache, float* v_cache, const float* k, const float* v,
                   int n_kv_heads, int head_dim, int max_seq, int pos);
void gbo_attention(const float* q, const float* k_cache, const float* v_cache,
                   int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos,
                   float* out);
void gbo_rmsnorm(const float* x, const float* w, float* out, int dim, float eps);
void gbo_silu_mul(float* gate, const float* up, int n);
int  gbo_argmax(const float* logits, int n);

/* One full decode layer, T = 1 (engine.c:353-554).  Weight dtypes use the
 * reference DataType codes (Q8_0 = 2, Q4_K = 4, Q6_K = 5).  hidden is in/out.
 * k_cache / v_cache are this layer's [n_kv][max_seq][head_dim] bases. */
typedef struct {
    const void* w[7];      /* wq, wk, wv, wo, gate, up, down */
    int rows[7], cols[7], dtype[7];
    const float* rms_att;
    const float* rms_ffn;
} gbo_layer_t;

int gbo_layer_decode(const gbo_layer_t* L, float* hidden, float* k_cache, float* v_cache,
                     int H, int n_heads, int n_kv_heads, int head_dim, int ff_dim,
                     int max_seq, int pos, float eps, float theta);

/* ---- seeded synthetic inputs (identical bytes on CPU and GPU) ----
 * Counter-based splitmix64: word i of stream s is mix64(seed + mix64(s + C) + (i+1)*G). */
uint64_t gbo_rand64(uint64_t seed, uint64_t stream, uint64_t i);
void gbo_synth_q4k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream);
void gbo_synth_q6k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream);
void gbo_synth_q8_0(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream);
void gbo_synth_q4k_at(uint8_t* blk, uint64_t b, uint64_t seed, uint64_t stream);
void gbo_synth_q5k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream);
void gbo_synth_f16(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream);
void gbo_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream);

#ifdef __cplusplus
}
#endif
#endif /* GB_ORACLE_H */
