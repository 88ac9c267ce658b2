/*
 * gb_backend.c -- C11 drop-in for src/backend/cuda_backend.c: builds the
 * KernelVTable whose quantised matvec slots run on the B200.
 *
 * Differences from the reference CUDA backend (cuda_backend.c:43-81):
 *  - the Q6_K and Q8_0 slots run on the GPU too (the reference left them on
 *    the CPU, cuda_backend.c:72-73);
 *  - a tensor without a device copy is uploaded once on first use instead of
 *    falling back to the CPU kernel (cuda_backend.c:36-38), which moves the
 *    lm_head matvec (engine.c:590) onto the GPU.
 * The non-quantised slots keep the engine's CPU kernels exactly as the
 * reference does; they are bound through weak references, so the library
 * also loads stand-alone (the slots are NULL then).
 */
#include "../../include/guanaco_backend_abi.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>

/* The engine's CPU kernels and thread pool (src/kernels/cpu/kernels_cpu.c,
 * src/threadpool/threadpool.c), resolved when linked into the engine. */
typedef struct ThreadPool ThreadPool;
extern void gemm_f32(const Tensor* A, const Tensor* B, Tensor* C) __attribute__((weak));
extern void gemm_f32_nn(const Tensor* A, const Tensor* B, Tensor* C) __attribute__((weak));
extern void cpu_rmsnorm(const Tensor* in, const Tensor* w, Tensor* out, float eps) __attribute__((weak));
extern void softmax_inplace(Tensor* scores, int seq_len) __attribute__((weak));
extern void silu_inplace(Tensor* x) __attribute__((weak));
extern void rope(Tensor* q, Tensor* k, int pos, int head_dim) __attribute__((weak));
extern void residual_add(Tensor* x, const Tensor* r) __attribute__((weak));
extern void elemwise_mul(Tensor* a, const Tensor* b) __attribute__((weak));
extern ThreadPool* threadpool_create(int n) __attribute__((weak));
extern void threadpool_destroy(ThreadPool* tp) __attribute__((weak));
extern void kernels_cpu_set_threadpool(ThreadPool* tp) __attribute__((weak));

/* gb_abi.cu */
extern int gb_vtable_matvec(int dtype, const void* host_data, const void* d_data, int resident, size_t byte_size,
                            int rows, int cols, const float* x, float* y);
extern int cuda_get_temperature(void);

/* Argument checks in the reference order (quant_matvec_q4_k.c:143-158). */
static int vt_matvec(DataType want, const Tensor* W, const float* x, float* y) {
    if (W == NULL || x == NULL || y == NULL) return -1;
    if (W->dtype != want || W->ndim != 2) return -1;
    return gb_vtable_matvec((int)want, W->data, W->d_data, W->device_residency, W->byte_size, W->shape[0],
                            W->shape[1], x, y);
}

int gb_backend_matvec_q4k_f32(const Tensor* W, const float* x, float* y) { return vt_matvec(DTYPE_Q4_K, W, x, y); }
int gb_backend_matvec_q6k_f32(const Tensor* W, const float* x, float* y) { return vt_matvec(DTYPE_Q6_K, W, x, y); }
int gb_backend_matvec_q8_0_f32(const Tensor* W, const float* x, float* y) { return vt_matvec(DTYPE_Q8_0, W, x, y); }

Backend* backend_cuda_create(const BackendConfig* cfg) {
    if (cfg == NULL) return NULL;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return NULL;
    if (cfg->device_id < 0 || cfg->device_id >= ndev) return NULL;
    if (cudaSetDevice(cfg->device_id) != cudaSuccess) return NULL;
    Backend* b = (Backend*)calloc(1, sizeof(Backend));
    if (!b) return NULL;
    b->cfg = *cfg;
    b->cfg.kind = BACKEND_CUDA;
    (void)cuda_get_temperature();   /* NVML set-up, as cuda_backend.c:51-55 */
    if (threadpool_create && kernels_cpu_set_threadpool) {
        ThreadPool* tp = threadpool_create(b->cfg.threads);
        b->impl = tp;
        kernels_cpu_set_threadpool(tp);
    }
    b->kernels.gemm_f32 = gemm_f32;
    b->kernels.gemm_f32_nn = gemm_f32_nn;
    b->kernels.rmsnorm = cpu_rmsnorm;
    b->kernels.softmax_inplace = softmax_inplace;
    b->kernels.silu_inplace = silu_inplace;
    b->kernels.rope = rope;
    b->kernels.residual_add = residual_add;
    b->kernels.elemwise_mul = elemwise_mul;
    b->kernels.matvec_q4k_f32 = gb_backend_matvec_q4k_f32;
    b->kernels.matvec_q6k_f32 = gb_backend_matvec_q6k_f32;
    b->kernels.matvec_q8_0_f32 = gb_backend_matvec_q8_0_f32;
    return b;
}

void backend_cuda_destroy(Backend* b) {
    if (!b) return;
    if (b->impl && threadpool_destroy && kernels_cpu_set_threadpool) {
        kernels_cpu_set_threadpool(NULL);
        threadpool_destroy((ThreadPool*)b->impl);
        b->impl = NULL;
    }
    free(b);
}
