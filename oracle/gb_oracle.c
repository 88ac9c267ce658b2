/*
 * gb_oracle.c -- CPU restatement of the Guanaco decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see gb_oracle.h).  Compiled with
 * `-std=c11 -O2 -ffp-contract=off` so that every a*b+c written below is two
 * roundings unless it is an explicit fmaf(), exactly like the reference's
 * gcc -std=c11 build.  Where the reference uses AVX2 FMA lanes the restatement
 * keeps eight scalar lanes and the same horizontal-sum order, which makes the
 * results bit-identical to the reference kernels, not merely close.
 */
#include "gb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Scalar helpers                                                            */
/* ------------------------------------------------------------------------ */

/* Restates extract_f16_to_f32 (src/kernels/cpu/quant_matvec_q4_k.c:18-45):
 * exact IEEE half -> float including subnormals, Inf and NaN payloads. */
float gbo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {                     /* subnormal: renormalise the mantissa */
            uint32_t e = 113;        /* 127 - 15 + 1 */
            while ((mant & 0x400u) == 0) { mant <<= 1; e--; }
            bits = sign | (e << 23) | ((mant & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE float -> half, round to nearest even (what __float2half_rn does).
 * Used only to build synthetic fp16 block scales identically on CPU and GPU. */
uint16_t gbo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                         /* Inf / NaN */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  /* rounds to Inf */
    if (ax < 0x38800000u) {                          /* half subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;                   /* 14..24 */
        uint32_t res = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (res & 1u))) res++;
        return (uint16_t)(sign | res);
    }
    uint32_t res = ((ax >> 13) - (112u << 10));
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (res & 1u))) res++;
    return (uint16_t)(sign | res);
}

/* Restates get_scale_min_k4 (src/kernels/cpu/quant_matvec_q4_k.c:47-56):
 * 8 six-bit scales and 8 six-bit mins packed into 12 bytes. */
void gbo_q4k_scale_min(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------------ */
/* Dequantisation                                                            */
/* ------------------------------------------------------------------------ */

/* Q4_K: restates the embedding dequantiser (src/engine/engine.c:248-276):
 * d1 = d*sc, m1 = dmin*m, w = d1*q - m1 with two roundings (no contraction). */
void gbo_dequant_q4k(const void* blocks, size_t nblocks, float* out) {
    const uint8_t* base = (const uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t* blk = base + b * GBO_Q4K_BYTES;
        const float d_all = gbo_f16_to_f32(rd16(blk));
        const float min_all = gbo_f16_to_f32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* q = blk + 16;
        float* px = out + b * 256;
        for (int g = 0; g < 4; g++) {
            uint8_t s, m;
            gbo_q4k_scale_min(2 * g, sc, &s, &m);
            const float d1 = d_all * s, m1 = min_all * m;
            gbo_q4k_scale_min(2 * g + 1, sc, &s, &m);
            const float d2 = d_all * s, m2 = min_all * m;
            for (int l = 0; l < 32; l++) px[l] = d1 * (q[l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) px[32 + l] = d2 * (q[l] >> 4) - m2;
            q += 32;
            px += 64;
        }
    }
}

/* Q6_K: the reference has no standalone Q6_K dequantiser; the weight value it
 * multiplies into x is (d * sc) * q, evaluated left to right
 * (src/kernels/cpu/quant_matvec_q6_k.c:75-92).  That product is the definition. */
void gbo_dequant_q6k(const void* blocks, size_t nblocks, float* out) {
    const uint8_t* base = (const uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t* blk = base + b * GBO_Q6K_BYTES;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        const float d_all = gbo_f16_to_f32(rd16(blk + 208));
        float* px = out + b * 256;
        for (int n = 0; n < 2; n++) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int8_t q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                px[l] = d_all * sc[is + 0] * q1;
                px[l + 32] = d_all * sc[is + 2] * q2;
                px[l + 64] = d_all * sc[is + 4] * q3;
                px[l + 96] = d_all * sc[is + 6] * q4;
            }
            px += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* Q8_0: restates src/engine/engine.c:235-240: w = q * scale. */
void gbo_dequant_q8_0(const void* blocks, size_t nblocks, float* out) {
    const uint8_t* base = (const uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t* blk = base + b * GBO_Q80_BYTES;
        const float scale = gbo_f16_to_f32(rd16(blk));
        const int8_t* qs = (const int8_t*)(blk + 2);
        for (int i = 0; i < 32; i++) out[b * 32 + i] = qs[i] * scale;
    }
}

/* Q5_K: the reference has no Q5_K kernel (its loader sizes the GGUF type,
 * src/engine/loader.c:98,117, and rejects it, :586-651).  Restated from GGML's
 * published k-quant layout (llama.cpp ggml-quants, block_q5_K {d, dmin,
 * scales[12], qh[32], qs[128]}, dequantize_row_q5_K): per 64 columns two
 * sub-blocks j = 2g, 2g + 1 with get_scale_min_k4 scales; q = low / high
 * nibble of qs[32 g + l] + 16 * bit j of qh[l]; w = (d sc) q - dmin m with two
 * roundings, as the reference's Q4_K dequantiser (engine.c:257-275). */
void gbo_dequant_q5k(const void* blocks, size_t nblocks, float* out) {
    const uint8_t* base = (const uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t* blk = base + b * GBO_Q5K_BYTES;
        const float d_all = gbo_f16_to_f32(rd16(blk));
        const float min_all = gbo_f16_to_f32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* q = blk + 48;
        float* px = out + b * 256;
        for (int g = 0; g < 4; g++) {
            uint8_t s, m;
            gbo_q4k_scale_min(2 * g, sc, &s, &m);
            const float d1 = d_all * s, m1 = min_all * m;
            gbo_q4k_scale_min(2 * g + 1, sc, &s, &m);
            const float d2 = d_all * s, m2 = min_all * m;
            for (int l = 0; l < 32; l++) px[l] = d1 * ((q[l] & 0xF) + ((qh[l] >> (2 * g)) & 1 ? 16 : 0)) - m1;
            for (int l = 0; l < 32; l++) px[32 + l] = d2 * ((q[l] >> 4) + ((qh[l] >> (2 * g + 1)) & 1 ? 16 : 0)) - m2;
            q += 32;
            px += 64;
        }
    }
}

/* F16 rows: each half converted exactly by the reference's own mapping
 * (extract_f16_to_f32, src/engine/engine.c:183-212); "blocks" of 32. */
void gbo_dequant_f16(const void* blocks, size_t nblocks, float* out) {
    const uint8_t* base = (const uint8_t*)blocks;
    for (size_t i = 0; i < nblocks * 32; i++) out[i] = gbo_f16_to_f32(rd16(base + 2 * i));
}

/* ------------------------------------------------------------------------ */
/* Matvec                                                                    */
/* ------------------------------------------------------------------------ */

/* Q4_K: restates matvec_q4k_cols / matvec_q4k_f32
 * (src/kernels/cpu/quant_matvec_q4_k.c:65-173).  The AVX2 loop keeps eight
 * FMA lanes per block: w = fmsub(d1, q, m1), lane += w * x; after the block
 * the eight lanes are summed left to right and added to the row sum. */
int gbo_matvec_q4k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y) {
    if (W == NULL || x == NULL || y == NULL) return -1;
    if (cols % 256 != 0) return -2;
    const int nb = cols / 256;
    if (byte_size != 0 && (size_t)rows * (size_t)nb * GBO_Q4K_BYTES > byte_size) return -3;
    const uint8_t* base = (const uint8_t*)W;
    for (int r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = base + ((size_t)r * nb + b) * GBO_Q4K_BYTES;
            const float d_all = gbo_f16_to_f32(rd16(blk));
            const float min_all = gbo_f16_to_f32(rd16(blk + 2));
            const uint8_t* q = blk + 16;
            const float* px = x + (size_t)b * 256;
            float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int g = 0; g < 4; g++) {
                uint8_t s, m;
                gbo_q4k_scale_min(2 * g, blk + 4, &s, &m);
                const float d1 = d_all * s, m1 = min_all * m;
                gbo_q4k_scale_min(2 * g + 1, blk + 4, &s, &m);
                const float d2 = d_all * s, m2 = min_all * m;
                for (int step = 0; step < 4; step++) {
                    for (int k = 0; k < 8; k++) {
                        const uint8_t qb = q[step * 8 + k];
                        const float w1 = fmaf(d1, (float)(qb & 0xF), -m1);
                        const float w2 = fmaf(d2, (float)(qb >> 4), -m2);
                        lane[k] = fmaf(w1, px[step * 8 + k], lane[k]);
                        lane[k] = fmaf(w2, px[32 + step * 8 + k], lane[k]);
                    }
                }
                q += 32;
                px += 64;
            }
            float t = lane[0];
            for (int k = 1; k < 8; k++) t += lane[k];
            sum += t;
        }
        y[r] = sum;
    }
    return 0;
}

/* Q6_K: restates matvec_q6k_f32 (src/kernels/cpu/quant_matvec_q6_k.c:43-98):
 * scalar, sum += ((d * sc) * q) * x, left to right, no contraction. */
int gbo_matvec_q6k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y) {
    if (W == NULL || x == NULL || y == NULL) return -1;
    if (cols % 256 != 0) return -2;
    const int nb = cols / 256;
    if (byte_size != 0 && (size_t)rows * (size_t)nb * GBO_Q6K_BYTES > byte_size) return -3;
    const uint8_t* base = (const uint8_t*)W;
    for (int r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = base + ((size_t)r * nb + b) * GBO_Q6K_BYTES;
            const float d_all = gbo_f16_to_f32(rd16(blk + 208));
            const uint8_t* ql = blk;
            const uint8_t* qh = blk + 128;
            const int8_t* sc = (const int8_t*)(blk + 192);
            const float* px = x + (size_t)b * 256;
            for (int n = 0; n < 2; n++) {
                for (int l = 0; l < 32; l++) {
                    const int is = l / 16;
                    const int8_t q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    sum += d_all * sc[is + 0] * q1 * px[l + 0];
                    sum += d_all * sc[is + 2] * q2 * px[l + 32];
                    sum += d_all * sc[is + 4] * q3 * px[l + 64];
                    sum += d_all * sc[is + 6] * q4 * px[l + 96];
                }
                px += 128;
                ql += 64;
                qh += 32;
                sc += 8;
            }
        }
        y[r] = sum;
    }
    return 0;
}

/* Q8_0: restates matvec_q8_0_f32 (src/kernels/cpu/quant_matvec_q8_0.c:41-78):
 * block_sum = sum q*x, then sum += block_sum * scale. */
int gbo_matvec_q8_0(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y) {
    if (W == NULL || x == NULL || y == NULL) return -1;
    if (cols % 32 != 0) return -2;
    const int nb = cols / 32;
    if (byte_size != 0 && (size_t)rows * (size_t)nb * GBO_Q80_BYTES > byte_size) return -3;
    const uint8_t* base = (const uint8_t*)W;
    for (int r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = base + ((size_t)r * nb + b) * GBO_Q80_BYTES;
            const float scale = gbo_f16_to_f32(rd16(blk));
            const int8_t* qs = (const int8_t*)(blk + 2);
            const float* px = x + (size_t)b * 32;
            float block_sum = 0.0f;
            for (int i = 0; i < 32; i++) block_sum += qs[i] * px[i];
            sum += block_sum * scale;
        }
        y[r] = sum;
    }
    return 0;
}

/* Q5_K / F16 (formats the reference does not compute): each row dequantised
 * by the definitions above, then dotted with x in 8 FMA lanes summed in the
 * order of the reference's gemm_f32 row dot (kernels_cpu.c:44-69).  Errors as
 * the reference kernels: -2 for columns not a multiple of the block width,
 * -3 when byte_size (if non-zero) is too small. */
static float dot_lanes(const float* a, const float* b, int K);
static int matvec_rows(int width, int bbytes, void (*deq)(const void*, size_t, float*), const void* W, int rows,
                       int cols, size_t byte_size, const float* x, float* y) {
    if (!W || !x || !y) return -1;
    if (cols % width) return -2;
    const size_t rb = (size_t)(cols / width) * bbytes;
    if (byte_size && rb * (size_t)rows > byte_size) return -3;
    float* w = (float*)malloc((size_t)cols * sizeof(float));
    if (!w) return -1;
    for (int r = 0; r < rows; r++) {
        deq((const uint8_t*)W + (size_t)r * rb, (size_t)(cols / width), w);
        y[r] = dot_lanes(w, x, cols);
    }
    free(w);
    return 0;
}
int gbo_matvec_q5k(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y) {
    return matvec_rows(256, GBO_Q5K_BYTES, gbo_dequant_q5k, W, rows, cols, byte_size, x, y);
}
int gbo_matvec_f16(const void* W, int rows, int cols, size_t byte_size, const float* x, float* y) {
    return matvec_rows(32, 64, gbo_dequant_f16, W, rows, cols, byte_size, x, y);
}

/* ------------------------------------------------------------------------ */
/* Decode-layer pieces                                                       */
/* ------------------------------------------------------------------------ */

/* Restates rope (src/kernels/cpu/kernels_cpu.c:391-431): interleaved pairs,
 * freq = 1/theta^(i/hd), all q heads then all k heads. */
void gbo_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos, float theta) {
    for (int i = 0; i < head_dim; i += 2) {
        const float freq = 1.0f / powf(theta, (float)i / (float)head_dim);
        const float angle = pos * freq;
        const float c = cosf(angle);
        const float s = sinf(angle);
        for (int h = 0; h < n_heads; h++) {
            float* p = q + (size_t)h * head_dim;
            const float a = p[i], b = p[i + 1];
            p[i] = a * c - b * s;
            p[i + 1] = a * s + b * c;
        }
        for (int h = 0; h < n_kv_heads; h++) {
            float* p = k + (size_t)h * head_dim;
            const float a = p[i], b = p[i + 1];
            p[i] = a * c - b * s;
            p[i + 1] = a * s + b * c;
        }
    }
}

/* Restates kv_cache_append (src/memory/kv_cache.c:90-128) for one layer whose
 * head-major cache base is given: slot = pos % max_seq. */
void gbo_kv_append(float* k_cache, float* v_cache, const float* k, const float* v,
                   int n_kv_heads, int head_dim, int max_seq, int pos) {
    const int slot = pos % max_seq;
    for (int h = 0; h < n_kv_heads; h++) {
        const size_t off = ((size_t)h * max_seq + slot) * head_dim;
        memcpy(k_cache + off, k + (size_t)h * head_dim, (size_t)head_dim * sizeof(float));
        memcpy(v_cache + off, v + (size_t)h * head_dim, (size_t)head_dim * sizeof(float));
    }
}

/* gemm_f32 row dot (src/kernels/cpu/kernels_cpu.c:44-69): 8 FMA lanes over the
 * 8-aligned prefix, lanes summed left to right, then an unfused scalar tail. */
static float dot_lanes(const float* a, const float* b, int K) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k <= K - 8; k += 8)
        for (int j = 0; j < 8; j++) lane[j] = fmaf(a[k + j], b[k + j], lane[j]);
    float sum = 0.0f;
    float t = lane[0];
    for (int j = 1; j < 8; j++) t += lane[j];
    sum += t;
    for (; k < K; k++) sum += a[k] * b[k];
    return sum;
}

/* Softmax over one row (src/kernels/cpu/kernels_cpu.c:271-310). */
static void softmax_row(float* x, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > max_val) max_val = x[i];
    if (isinf(max_val) && max_val < 0) {
        for (int i = 0; i < n; i++) x[i] = 0.0f;
        return;
    }
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    if (sum < 1e-10f) sum = 1e-10f;
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* GQA single-query attention, restating src/engine/engine.c:433-509 for T = 1:
 * scores = gemm_f32(q_h, K_kvh); *scale after the dot; mask s > pos;
 * softmax; ctx = gemm_f32_nn(p, V_kvh) (8-lane FMA over k for the 8-aligned
 * column prefix, kernels_cpu.c:91-111).  seq_len = pos + 1 <= max_seq. */
void gbo_attention(const float* q, const float* k_cache, const float* v_cache,
                   int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos,
                   float* out) {
    const int seq_len = pos + 1;
    const int group = n_heads / n_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float* scores = (float*)malloc((size_t)seq_len * sizeof(float));
    const int vec_cols = head_dim - head_dim % 8;
    for (int h = 0; h < n_heads; h++) {
        const int kvh = h / group;
        const float* qh = q + (size_t)h * head_dim;
        const float* kh = k_cache + (size_t)kvh * max_seq * head_dim;
        const float* vh = v_cache + (size_t)kvh * max_seq * head_dim;
        for (int s = 0; s < seq_len; s++) {
            float v = dot_lanes(qh, kh + (size_t)s * head_dim, head_dim) * scale;
            if (s > pos) v = -INFINITY;
            scores[s] = v;
        }
        softmax_row(scores, seq_len);
        float* o = out + (size_t)h * head_dim;
        for (int j = 0; j < vec_cols; j++) {          /* vector columns: FMA chain */
            float acc = 0.0f;
            for (int s = 0; s < seq_len; s++) acc = fmaf(scores[s], vh[(size_t)s * head_dim + j], acc);
            o[j] = acc;
        }
        for (int j = vec_cols; j < head_dim; j++) {   /* scalar tail: unfused */
            float acc = 0.0f;
            for (int s = 0; s < seq_len; s++) acc += scores[s] * vh[(size_t)s * head_dim + j];
            o[j] = acc;
        }
    }
    free(scores);
}

/* Restates cpu_rmsnorm (src/kernels/cpu/kernels_cpu.c:199-265). */
void gbo_rmsnorm(const float* x, const float* w, float* out, int dim, float eps) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j <= dim - 8; j += 8)
        for (int k = 0; k < 8; k++) lane[k] = fmaf(x[j + k], x[j + k], lane[k]);
    float ss = lane[0];
    for (int k = 1; k < 8; k++) ss += lane[k];
    for (; j < dim; j++) ss += x[j] * x[j];
    ss /= dim;
    ss += eps;
    ss = 1.0f / sqrtf(ss);
    for (j = 0; j < dim; j++) out[j] = (w ? w[j] : 1.0f) * (x[j] * ss);
}

/* silu_inplace then elemwise_mul (src/kernels/cpu/kernels_cpu.c:312-389):
 * vector lanes use x * (1/(1+exp(-x))), the scalar tail x / (1+exp(-x)). */
void gbo_silu_mul(float* gate, const float* up, int n) {
    int i = 0;
    for (; i <= n - 8; i += 8)
        for (int k = 0; k < 8; k++) {
            const float g = gate[i + k];
            const float sig = 1.0f / (1.0f + expf(-g));
            gate[i + k] = g * sig;
        }
    for (; i < n; i++) gate[i] = gate[i] / (1.0f + expf(-gate[i]));
    for (i = 0; i < n; i++) gate[i] *= up[i];
}

/* Restates sample_greedy (src/tokenizer/tokenizer.c:175-185): the first
 * maximum wins (strict >). */
int gbo_argmax(const float* logits, int n) {
    int best = 0;
    float best_val = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > best_val) { best_val = logits[i]; best = i; }
    return best;
}

static int matvec_any(int dtype, const void* W, int rows, int cols, const float* x, float* y) {
    switch (dtype) {
        case 2: return gbo_matvec_q8_0(W, rows, cols, 0, x, y);
        case 4: return gbo_matvec_q4k(W, rows, cols, 0, x, y);
        case 5: return gbo_matvec_q6k(W, rows, cols, 0, x, y);
        case GBO_DT_Q5_K: return gbo_matvec_q5k(W, rows, cols, 0, x, y);
        case 1: return gbo_matvec_f16(W, rows, cols, 0, x, y);
        default: return -1;
    }
}

/* One decode layer (T = 1) in the order of src/engine/engine.c:353-554. */
int gbo_layer_decode(const gbo_layer_t* L, float* hidden, float* k_cache, float* v_cache,
                     int H, int n_heads, int n_kv_heads, int head_dim, int ff_dim,
                     int max_seq, int pos, float eps, float theta) {
    if (pos < 0 || pos >= max_seq) return -4;
    const int kv_dim = n_kv_heads * head_dim;
    float* residual = (float*)malloc((size_t)H * 4);
    float* normed = (float*)malloc((size_t)H * 4);
    float* Q = (float*)malloc((size_t)n_heads * head_dim * 4);
    float* K = (float*)malloc((size_t)kv_dim * 4);
    float* V = (float*)malloc((size_t)kv_dim * 4);
    float* attn = (float*)malloc((size_t)n_heads * head_dim * 4);
    float* proj = (float*)malloc((size_t)H * 4);
    float* gate = (float*)malloc((size_t)ff_dim * 4);
    float* up = (float*)malloc((size_t)ff_dim * 4);
    int rc = 0;
    memcpy(residual, hidden, (size_t)H * 4);
    gbo_rmsnorm(hidden, L->rms_att, normed, H, eps);
    rc |= matvec_any(L->dtype[0], L->w[0], L->rows[0], L->cols[0], normed, Q);
    rc |= matvec_any(L->dtype[1], L->w[1], L->rows[1], L->cols[1], normed, K);
    rc |= matvec_any(L->dtype[2], L->w[2], L->rows[2], L->cols[2], normed, V);
    gbo_rope(Q, K, n_heads, n_kv_heads, head_dim, pos, theta);
    gbo_kv_append(k_cache, v_cache, K, V, n_kv_heads, head_dim, max_seq, pos);
    gbo_attention(Q, k_cache, v_cache, n_heads, n_kv_heads, head_dim, max_seq, pos, attn);
    rc |= matvec_any(L->dtype[3], L->w[3], L->rows[3], L->cols[3], attn, proj);
    for (int i = 0; i < H; i++) proj[i] += residual[i];
    memcpy(residual, proj, (size_t)H * 4);
    gbo_rmsnorm(proj, L->rms_ffn, normed, H, eps);
    rc |= matvec_any(L->dtype[4], L->w[4], L->rows[4], L->cols[4], normed, gate);
    rc |= matvec_any(L->dtype[5], L->w[5], L->rows[5], L->cols[5], normed, up);
    gbo_silu_mul(gate, up, ff_dim);
    rc |= matvec_any(L->dtype[6], L->w[6], L->rows[6], L->cols[6], gate, hidden);
    for (int i = 0; i < H; i++) hidden[i] += residual[i];
    free(residual); free(normed); free(Q); free(K); free(V);
    free(attn); free(proj); free(gate); free(up);
    return rc ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs (counter-based splitmix64; pure integer and exact  */
/* float arithmetic, so the CUDA generator reproduces the same bytes)         */
/* ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t gbo_rand64(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(seed + mix64(stream + 0x632BE59BD9B4E019ull) + (i + 1) * 0x9E3779B97F4A7C15ull);
}

/* fp16 of U[1e-4, 1e-3] from 24 random bits: 1e-4 + u * 9e-4, two roundings. */
static uint16_t synth_scale(uint64_t bits24) {
    const float u = (float)(bits24 & 0xffffffu) * (1.0f / 16777216.0f);
    const float v = 1e-4f + u * 9e-4f;
    return gbo_f32_to_f16(v);
}

static inline void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* Q4_K block: d, dmin ~ fp16 U[1e-4,1e-3]; 8 scales and 8 mins U{0..63}
 * packed as get_scale_min_k4 unpacks them; qs uniform bytes (two U{0..15}). */
void gbo_synth_q4k_at(uint8_t* blk, uint64_t b, uint64_t seed, uint64_t stream) {
    const uint64_t i0 = b * 32;
    const uint64_t r0 = gbo_rand64(seed, stream, i0);
    wr16(blk, synth_scale(r0));
    wr16(blk + 2, synth_scale(r0 >> 24));
    const uint64_t r1 = gbo_rand64(seed, stream, i0 + 1);
    const uint64_t r2 = gbo_rand64(seed, stream, i0 + 2);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)((r1 >> (6 * j)) & 63);
        mn[j] = (uint8_t)((r2 >> (6 * j)) & 63);
    }
    uint8_t* s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
    for (int w = 0; w < 16; w++) {
        const uint64_t r = gbo_rand64(seed, stream, i0 + 3 + w);
        memcpy(blk + 16 + 8 * w, &r, 8);
    }
}

void gbo_synth_q4k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream) {
    uint8_t* base = (uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) gbo_synth_q4k_at(base + b * GBO_Q4K_BYTES, (uint64_t)b, seed, stream);
}

/* Q6_K block: ql, qh uniform bytes; scales int8 U{-32..31}; d fp16 U[1e-4,1e-3]. */
void gbo_synth_q6k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream) {
    uint8_t* base = (uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        uint8_t* blk = base + b * GBO_Q6K_BYTES;
        const uint64_t i0 = (uint64_t)b * 32;
        for (int w = 0; w < 24; w++) {              /* ql[128] then qh[64] */
            const uint64_t r = gbo_rand64(seed, stream, i0 + w);
            memcpy(blk + 8 * w, &r, 8);
        }
        const uint64_t r1 = gbo_rand64(seed, stream, i0 + 24);
        const uint64_t r2 = gbo_rand64(seed, stream, i0 + 25);
        for (int j = 0; j < 16; j++) {
            const uint64_t r = j < 8 ? r1 : r2;
            blk[192 + j] = (uint8_t)(int8_t)((int)((r >> (6 * (j & 7))) & 63) - 32);
        }
        wr16(blk + 208, synth_scale(gbo_rand64(seed, stream, i0 + 26)));
    }
}

/* Q8_0 block: scale fp16 U[1e-4,1e-3]; 32 uniform int8 quants. */
void gbo_synth_q8_0(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream) {
    uint8_t* base = (uint8_t*)blocks;
    for (size_t b = 0; b < nblocks; b++) {
        uint8_t* blk = base + b * GBO_Q80_BYTES;
        const uint64_t i0 = (uint64_t)b * 8;
        wr16(blk, synth_scale(gbo_rand64(seed, stream, i0)));
        for (int w = 0; w < 4; w++) {
            const uint64_t r = gbo_rand64(seed, stream, i0 + 1 + w);
            memcpy(blk + 2 + 8 * w, &r, 8);
        }
    }
}

/* Q5_K block: the Q4_K block's header and nibbles (same random words), then
 * 32 bytes of fifth bits from words 19-22. */
void gbo_synth_q5k(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream) {
    uint8_t* base = (uint8_t*)blocks;
    uint8_t tmp[GBO_Q4K_BYTES];
    for (size_t b = 0; b < nblocks; b++) {
        uint8_t* blk = base + b * GBO_Q5K_BYTES;
        /* the Q4_K generator for global block b of this stream */
        const uint64_t i0 = (uint64_t)b * 32;
        gbo_synth_q4k_at(tmp, (uint64_t)b, seed, stream);
        memcpy(blk, tmp, 16);
        for (int w = 0; w < 4; w++) {
            const uint64_t r = gbo_rand64(seed, stream, i0 + 19 + w);
            memcpy(blk + 16 + 8 * w, &r, 8);
        }
        memcpy(blk + 48, tmp + 16, 128);
    }
}

/* F16 "blocks" of 32 halves: the Irwin-Hall value of gbo_synth_normal at
 * index i, times 2^-5, rounded to the nearest half (ties to even). */
void gbo_synth_f16(void* blocks, size_t nblocks, uint64_t seed, uint64_t stream) {
    uint8_t* base = (uint8_t*)blocks;
    for (size_t i = 0; i < nblocks * 32; i++) {
        int32_t acc = 0;
        for (int w = 0; w < 3; w++) {
            const uint64_t r = gbo_rand64(seed, stream, 3 * (uint64_t)i + w);
            acc += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) +
                   (int32_t)((r >> 32) & 0xffff) + (int32_t)((r >> 48) & 0xffff);
        }
        wr16(base + 2 * i, gbo_f32_to_f16((float)(acc + 6 - 393216) * (1.0f / 2097152.0f)));
    }
}

/* Approximately N(0,1): Irwin-Hall sum of twelve 16-bit uniforms, done in
 * integers and scaled by 2^-16, so the value is exact on any IEEE machine.
 * Mean 0, variance 1, support (-6, 6). */
void gbo_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream) {
    for (size_t i = 0; i < n; i++) {
        int32_t acc = 0;
        for (int w = 0; w < 3; w++) {
            const uint64_t r = gbo_rand64(seed, stream, 3 * (uint64_t)i + w);
            acc += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) +
                   (int32_t)((r >> 32) & 0xffff) + (int32_t)((r >> 48) & 0xffff);
        }
        out[i] = (float)(acc + 6 - 393216) * (1.0f / 65536.0f);
    }
}
