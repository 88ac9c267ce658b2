/*
 * guanaco_backend_abi.h -- the Guanaco backend types that the drop-in vtable
 * factory exchanges with the unchanged engine, laid out field for field as
 * the reference defines them:
 *   Tensor, DataType      src/include/types.h:16-62
 *   BackendKind/Config    src/include/backend.h:13-46
 *   KernelVTable          src/include/backend.h:21-39
 *   struct Backend        src/backend/backend_internal.h:7-11
 * A maintainer building the reference with this library compiles
 * gb_backend.c with -DGB_USE_REFERENCE_HEADERS -I<guanaco>/src/include so the
 * reference's own headers are used; this file is the stand-alone equivalent
 * (tests/test_abi.py checks its offsets against a fixture taken from the
 * reference headers).
 */
#ifndef GUANACO_BACKEND_ABI_H
#define GUANACO_BACKEND_ABI_H

#ifdef GB_USE_REFERENCE_HEADERS
#include "backend_internal.h"
#else

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    DTYPE_F32 = 0,
    DTYPE_F16 = 1,
    DTYPE_Q8_0 = 2,
    DTYPE_Q4_0 = 3,
    DTYPE_Q4_K = 4,
    DTYPE_Q6_K = 5,
    DTYPE_UNKNOWN = 99,
} DataType;

#define MAX_DIMS 4

typedef struct {
    void* data;               /* host bytes (GGUF mmap for weights) */
    int shape[MAX_DIMS];      /* shape[0] = rows (out features) */
    int stride[MAX_DIMS];     /* in elements */
    int ndim;
    DataType dtype;
    uint32_t ggml_type;
    size_t byte_size;         /* authoritative size for quantised tensors, 0 if unknown */
    int device_residency;     /* 1 when d_data holds a device copy */
    void* d_data;
} Tensor;

typedef enum { BACKEND_AUTO = -1, BACKEND_CPU = 0, BACKEND_CUDA = 1 } BackendKind;

typedef struct Backend Backend;

typedef struct {
    void (*gemm_f32)(const Tensor* A, const Tensor* B, Tensor* C);
    void (*gemm_f32_nn)(const Tensor* A, const Tensor* B, Tensor* C);
    void (*rmsnorm)(const Tensor* input, const Tensor* weight, Tensor* output, float eps);
    void (*softmax_inplace)(Tensor* scores, int seq_len);
    void (*silu_inplace)(Tensor* x);
    void (*rope)(Tensor* q, Tensor* k, int pos, int head_dim);
    void (*residual_add)(Tensor* x, const Tensor* residual);
    void (*elemwise_mul)(Tensor* a, const Tensor* b);
    int (*matvec_q4k_f32)(const Tensor* W_q4k, const float* x, float* y);
    int (*matvec_q6k_f32)(const Tensor* W_q6k, const float* x, float* y);
    int (*matvec_q8_0_f32)(const Tensor* W_q8_0, const float* x, float* y);
} KernelVTable;

typedef struct {
    BackendKind kind;
    int threads;
    int device_id;
    int n_gpu_layers;
} BackendConfig;

struct Backend {
    BackendConfig cfg;
    KernelVTable kernels;
    void* impl;
};

#ifdef __cplusplus
}
#endif
#endif /* GB_USE_REFERENCE_HEADERS */

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces backend_cuda_create / backend_cuda_destroy
 * (src/backend/cuda_backend.c:43-97, declared backend_internal.h:16-17).
 * The three quantised matvec slots run on the B200 for every tensor:
 * device-resident ones use W->d_data, others are uploaded once on first use
 * (lm_head is never uploaded by the reference loader).  The other slots keep
 * the engine's CPU kernels, as the reference CUDA backend does
 * (cuda_backend.c:62-69).  Returns NULL when no CUDA device is usable. */
Backend* backend_cuda_create(const BackendConfig* cfg);
void backend_cuda_destroy(Backend* b);

/* The vtable's quantised slots, exported for tests and callers that build
 * their own tables.  Same signatures and return codes as
 * src/kernels/cpu/quant_matvec_q4_k.c:142-173 and friends. */
int gb_backend_matvec_q4k_f32(const Tensor* W, const float* x, float* y);
int gb_backend_matvec_q6k_f32(const Tensor* W, const float* x, float* y);
int gb_backend_matvec_q8_0_f32(const Tensor* W, const float* x, float* y);

#ifdef __cplusplus
}
#endif
#endif /* GUANACO_BACKEND_ABI_H */
