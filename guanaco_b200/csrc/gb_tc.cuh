// gb_tc.cuh -- 5th-generation tensor core (tcgen05) building blocks for the
// prefill GEMMs on sm_100a: tensor-memory allocation, shared-memory matrix
// descriptors, the MMA instruction descriptor, MMA issue and completion
// tracking, and tensor-memory loads.
//
// Operand layout used here: K-major, no swizzle.  A tile of R rows x 32
// fp32 / tf32 elements is stored as "core matrices" of 8 rows x 4 elements
// (16 bytes per row, 128 bytes each): element (r, k) lives at
//     (r / 8) * 128 + (k / 4) * (R / 8 * 128) + (r % 8) * 16 + (k % 4) * 4
// bytes from the tile base, so consecutive 8-row groups are 128 bytes apart
// (the descriptor's stride byte offset) and consecutive 4-element column
// groups R * 16 bytes apart (its leading byte offset).  One tf32 MMA covers
// K = 8, i.e. two column groups.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gb {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Byte offset of element (r, k) in a K-major tile of R rows x 32 elements.
__host__ __device__ __forceinline__ uint32_t tile_off(int r, int k, int R) {
    return (uint32_t)((r >> 3) * 128 + (k >> 2) * (R / 8 * 128) + (r & 7) * 16 + (k & 3) * 4);
}

// The same layout for 16-bit elements: core matrices of 8 rows x 8 elements
// (still 16 bytes per row), so one f16 MMA (K = 16) also covers two column
// groups and the descriptors are unchanged.
__host__ __device__ __forceinline__ uint32_t tile_off16(int r, int k, int R) {
    return (uint32_t)((r >> 3) * 128 + (k >> 3) * (R / 8 * 128) + (r & 7) * 16 + (k & 7) * 2);
}

// Shared-memory matrix descriptor (sm_100): start address, leading byte
// offset (between core matrices along K) and stride byte offset (between
// 8-row groups), each in 16-byte units; descriptor version 1; no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;   // version
    return d;                 // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::tf32 with fp32 accumulation, both operands
// K-major, M x N (M = 128, N a multiple of 16 up to 256).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4)                        // D format: f32
         | (2u << 7)                        // A format: tf32
         | (2u << 10)                       // B format: tf32
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Instruction descriptor of kind::f16 with fp16 A and B (the same type, as
// the instruction requires) and fp32 accumulation, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                        // D format: f32
         | (0u << 7)                        // A format: f16
         | (0u << 10)                       // B format: f16
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

// Tensor memory: a warp allocates ncols columns (a power of two >= 32) and
// writes the base address to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes made visible to the tensor cores (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[smem] . B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T with fp16 operands (K = 16 per instruction).
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T: A (M rows = lanes, K columns of 32-bit
// elements) read from tensor memory at a_tmem, issued by one thread.
__device__ __forceinline__ void mma_tf32_ta(uint32_t tmem_d, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// Arrive once on an mbarrier when every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 16 consecutive fp32 columns of this thread's tensor-memory lane (warp w of
// a warpgroup reads lanes 32 (w % 4) .. + 31; taddr carries the lane in bits
// 31:16 and the column in 15:0).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive fp32 columns at each of two tensor-memory addresses of this
// thread's lane (same lane rule as tmem_ld16), one wait for both.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, float (&va)[32], float (&vb)[32]) {
    uint32_t a[32], b[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]), "=r"(a[24]), "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), "=r"(a[31]),
          "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15]), "=r"(b[16]), "=r"(b[17]), "=r"(b[18]), "=r"(b[19]), "=r"(b[20]), "=r"(b[21]), "=r"(b[22]), "=r"(b[23]), "=r"(b[24]), "=r"(b[25]), "=r"(b[26]), "=r"(b[27]), "=r"(b[28]), "=r"(b[29]), "=r"(b[30]), "=r"(b[31])
        : "r"(ta), "r"(tb)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) {
        va[i] = __uint_as_float(a[i]);
        vb[i] = __uint_as_float(b[i]);
    }
}
// 32 consecutive fp32 columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t ta, float (&va)[32]) {
    uint32_t a[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]), "=r"(a[24]), "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), "=r"(a[31])
        : "r"(ta)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) va[i] = __uint_as_float(a[i]);
}
// Store 32 consecutive fp32 columns of this thread's lane without waiting
// for completion (tmem_wait_st before the columns are read again).
__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Store 16 consecutive fp32 columns of this thread's tensor-memory lane
// (same lane rule as tmem_ld16), then wait for the store to complete.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// x = hi + lo with hi representable in tf32 (the top 19 bits, rounded to
// nearest with ties away from zero: half a tf32 unit added to the magnitude
// bits, then the low 13 bits cleared -- two integer operations instead of a
// conversion) and lo = x - hi exact in fp32; the tensor core reads lo as
// tf32 too, so hi.hi + hi.lo + lo.hi carries ~22 bits of each operand.
// Finite inputs only (a magnitude within half a unit of FLT_MAX rounds to inf).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = x - hi;
}

// Two values split for fp16 operands: the 11-bit hi of split_tf32 is exact in
// fp16 (for magnitudes in its normal range; callers scale by powers of two
// so that |x| < 2^15), and the fp32 remainder is rounded to fp16.  Returns
// the packed hi pair (first value in the low half) and the lo pair.
__device__ __forceinline__ void split_f16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
    float ha, la, hb, lb;
    split_tf32(a, ha, la);
    split_tf32(b, hb, lb);
    const __half2 h = __floats2half2_rn(ha, hb), l = __floats2half2_rn(la, lb);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Power-of-two exponent e for which 2^e * m lies in [2^14, 2^15), from the
// bits of a magnitude m >= 0: 0 for inf / NaN, the largest (126) for zero and
// fp32 subnormals; clamped to [-126, 126] so that 2^e and 2^-e are both
// normal floats.
__host__ __device__ __forceinline__ int f16_scale_exp(uint32_t mbits) {
    const int E = (int)((mbits >> 23) & 0xFFu);
    if (E == 255) return 0;
    if (E == 0) return 126;
    const int e = 141 - E;
    return e < -126 ? -126 : (e > 126 ? 126 : e);
}
// 2^e for |e| <= 126, built from its exponent bits.
__device__ __forceinline__ float pow2f(int e) {
    return __uint_as_float((uint32_t)(127 + e) << 23);
}

// Byte e (0..3) of w as an exact float minus `bias`: the byte is placed in
// the low mantissa bits of 2^23 by one byte permute, and 2^23 + bias is
// subtracted (exact for bytes and small integer biases).
template <int E>
__device__ __forceinline__ float byte_as_float(uint32_t w, float bias) {
    const uint32_t f = __byte_perm(w, 0x4B000000u, (uint32_t)E | 0x7540u);   // bytes {w.E, 0, 0, 0x4B}
    return __uint_as_float(f) - (8388608.0f + bias);
}

}  // namespace tc
}  // namespace gb
