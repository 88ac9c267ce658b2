// gb_common.cuh -- shared definitions for the sm_100a decode-path kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// Reference DataType codes (src/include/types.h:16-24).
#define GB_DT_F32 0
#define GB_DT_F16 1
#define GB_DT_Q8_0 2
#define GB_DT_Q4_K 4
#define GB_DT_Q6_K 5
// Q5_K has no code in the reference's DataType (its loader sizes the GGUF
// type, src/engine/loader.c:98,117, and rejects it, :586-651); 13 is its
// GGML type number.
#define GB_DT_Q5_K 13

// GGUF block sizes (src/engine/loader.c:113-119).
#define GB_Q4K_BYTES 144
#define GB_Q6K_BYTES 210
#define GB_Q80_BYTES 34
#define GB_Q5K_BYTES 176
// F16 rows are handled in "blocks" of 32 halves (64 bytes).
#define GB_F16_BYTES 64

// Error codes shared by every entry point.  0..-3 follow the reference vtable
// convention (src/kernels/cpu/quant_matvec_q4_k.c:143-158); the rest are new.
#define GB_OK 0
#define GB_EINVAL -1      // NULL pointer, bad dtype / ndim
#define GB_ESHAPE -2      // cols not a multiple of the block width
#define GB_ESIZE -3       // byte_size too small for rows x cols
#define GB_EPOS -4        // position outside [0, max_seq)
#define GB_ECUDA -5       // a CUDA runtime call failed
#define GB_ENOMEM -6      // device allocation failed
#define GB_ETIMEOUT -7    // a bounded device-side wait ran out
#define GB_ELIMIT -8      // size above a documented maximum

// Upper bound on the SM count of a device (B200: 148); buffers sized per SM
// use it, grids use the device's own count (gb::sm_count()).
#define GB_MAX_SMS 192

#define GB_CUDA_TRY(expr)                                   \
    do {                                                    \
        cudaError_t gb_err__ = (expr);                      \
        if (gb_err__ != cudaSuccess) return GB_ECUDA;       \
    } while (0)

static inline size_t gb_block_bytes(int dtype) {
    return dtype == GB_DT_Q4_K ? GB_Q4K_BYTES
         : dtype == GB_DT_Q6_K ? GB_Q6K_BYTES
         : dtype == GB_DT_Q8_0 ? GB_Q80_BYTES
         : dtype == GB_DT_Q5_K ? GB_Q5K_BYTES
         : dtype == GB_DT_F16 ? GB_F16_BYTES : 0;
}
static inline int gb_block_width(int dtype) { return dtype == GB_DT_Q8_0 || dtype == GB_DT_F16 ? 32 : 256; }
static inline size_t gb_matrix_bytes(int dtype, int rows, int cols) {
    return (size_t)rows * (size_t)(cols / gb_block_width(dtype)) * gb_block_bytes(dtype);
}

// ---------------------------------------------------------------- device side
namespace gb {

// Exact IEEE half -> float by bit manipulation (NaN payloads kept), the same
// mapping as the reference's extract_f16_to_f32 (quant_matvec_q4_k.c:18-45).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            const int lz = __clz(m) - 21;          // shifts that bring bit 10 up
            m = (m << lz) & 0x3ffu;
            bits = sign | ((uint32_t)(113 - lz) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

// Read-only 128-bit / 32-bit / 16-bit global loads through the non-coherent path.
__device__ __forceinline__ uint4 ldg4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint32_t ldg1(const void* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }
__device__ __forceinline__ uint32_t ldg_u16(const void* p) {
    return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
}

// Streaming 128-bit load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg4_stream(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// An integer bit pattern below 2^24 read as a float is exactly
// pattern * 2^-149 (subnormals and the first normal binade are linear).
// Masking a field in place therefore yields field * 2^(shift - 149) with a
// single LOP; the matching x element carries the compensating 2^(100 - shift),
// so products land at field * x * 2^-49 and the caller rescales by 2^49.
__device__ __forceinline__ float lin(uint32_t bits) { return __uint_as_float(bits); }

// Byte 3 of w moved to byte 2 (everything else zero): keeps field bits below 2^24.
__device__ __forceinline__ uint32_t b3_to_b2(uint32_t w) { return __byte_perm(w, 0u, 0x4344u); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

}  // namespace gb
