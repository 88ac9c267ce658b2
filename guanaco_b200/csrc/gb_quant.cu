// gb_quant.cu -- bit-exact GGUF dequantisers (Q4_K / Q6_K / Q8_0 / Q5_K / F16) and the
// seeded synthetic block / activation generators used by the tests and the
// benchmark.  The fused dequant + matvec kernels live in gb_matvec.cu.
//
// Dequantisation semantics (the value the reference multiplies into x):
//   Q4_K  src/engine/engine.c:257-275   w = (d*sc)*q - dmin*m, two roundings
//   Q6_K  src/kernels/cpu/quant_matvec_q6_k.c:84-87   w = (d*sc)*(q-32)
//   Q8_0  src/engine/engine.c:238       w = q*scale
//   Q5_K  (GGML k-quant; no reference kernel) w = (d*sc)*q - dmin*m, q = nibble
//         + 16 x bit j of qh for sub-block j, two roundings like Q4_K
//   F16   exact half -> float (engine.c:183-212's mapping)
#include "gb_common.cuh"
#include "gb_internal.h"

namespace gb {

// ------------------------------------------------------------------ dequant
// Bit-exact dequantisers (one thread per output pair / element).
__global__ void k_dequant_q4k(const uint8_t* __restrict__ B, size_t nblocks, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // one qs byte
    if (i >= nblocks * 128) return;
    const size_t b = i >> 7;
    const int l = (int)(i & 127), g = l >> 5, ll = l & 31;
    const uint8_t* blk = B + b * GB_Q4K_BYTES;
    const float d_all = f16_bits_to_f32(blk[0] | (blk[1] << 8));
    const float min_all = f16_bits_to_f32(blk[2] | (blk[3] << 8));
    const uint8_t* s = blk + 4;
    uint32_t sc[2], mn[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = 2 * g + h;
        if (j < 4) { sc[h] = s[j] & 63; mn[h] = s[j + 4] & 63; }
        else {
            sc[h] = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
            mn[h] = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
    }
    const uint8_t q = blk[16 + l];
    float* o = out + b * 256 + 64 * g;
    // engine.c:259-270: d1 = d*sc, m1 = dmin*m, w = d1*q - m1 (two roundings)
    o[ll] = __fsub_rn(__fmul_rn(__fmul_rn(d_all, (float)sc[0]), (float)(q & 0xF)), __fmul_rn(min_all, (float)mn[0]));
    o[32 + ll] = __fsub_rn(__fmul_rn(__fmul_rn(d_all, (float)sc[1]), (float)(q >> 4)), __fmul_rn(min_all, (float)mn[1]));
}

__global__ void k_dequant_q6k(const uint8_t* __restrict__ B, size_t nblocks, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // one (n, l)
    if (i >= nblocks * 64) return;
    const size_t b = i >> 6;
    const int n = (int)((i >> 5) & 1), l = (int)(i & 31), is = l >> 4;
    const uint8_t* blk = B + b * GB_Q6K_BYTES;
    const uint8_t* ql = blk + 64 * n;
    const uint8_t qh = blk[128 + 32 * n + l];
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * n);
    const float d_all = f16_bits_to_f32(blk[208] | (blk[209] << 8));
    const int q1 = (int)((ql[l] & 0xF) | (((qh >> 0) & 3) << 4)) - 32;
    const int q2 = (int)((ql[l + 32] & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
    const int q3 = (int)((ql[l] >> 4) | (((qh >> 4) & 3) << 4)) - 32;
    const int q4 = (int)((ql[l + 32] >> 4) | (((qh >> 6) & 3) << 4)) - 32;
    float* o = out + b * 256 + 128 * n;
    // (d * sc) * q, left to right (quant_matvec_q6_k.c:84-87)
    o[l] = __fmul_rn(__fmul_rn(d_all, (float)sc[is]), (float)q1);
    o[l + 32] = __fmul_rn(__fmul_rn(d_all, (float)sc[is + 2]), (float)q2);
    o[l + 64] = __fmul_rn(__fmul_rn(d_all, (float)sc[is + 4]), (float)q3);
    o[l + 96] = __fmul_rn(__fmul_rn(d_all, (float)sc[is + 6]), (float)q4);
}

__global__ void k_dequant_q8_0(const uint8_t* __restrict__ B, size_t nblocks, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks * 32) return;
    const uint8_t* blk = B + (i >> 5) * GB_Q80_BYTES;
    const float scale = f16_bits_to_f32(blk[0] | (blk[1] << 8));
    out[i] = __fmul_rn((float)(int8_t)blk[2 + (i & 31)], scale);   // engine.c:238
}

__global__ void k_dequant_q5k(const uint8_t* __restrict__ B, size_t nblocks, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // one qs byte
    if (i >= nblocks * 128) return;
    const size_t b = i >> 7;
    const int l = (int)(i & 127), g = l >> 5, ll = l & 31;
    const uint8_t* blk = B + b * GB_Q5K_BYTES;
    const float d_all = f16_bits_to_f32(blk[0] | (blk[1] << 8));
    const float min_all = f16_bits_to_f32(blk[2] | (blk[3] << 8));
    const uint8_t* s = blk + 4;
    const uint8_t qh = blk[16 + ll], q = blk[48 + l];
    float* o = out + b * 256 + 64 * g;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = 2 * g + h;
        uint32_t sc, mn;
        if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
        else {
            sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
            mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const uint32_t code = ((q >> (4 * h)) & 0xF) | (((qh >> j) & 1) << 4);
        o[32 * h + ll] = __fsub_rn(__fmul_rn(__fmul_rn(d_all, (float)sc), (float)code), __fmul_rn(min_all, (float)mn));
    }
}

__global__ void k_dequant_f16(const uint16_t* __restrict__ B, size_t n, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = f16_bits_to_f32(B[i]);
}

// ------------------------------------------------------------------ synthesis
// Device twin of the CPU generators the tests check against: same counter-based
// splitmix64 words, same packing, same float roundings, so the bytes match.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t rand64(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(seed + mix64(stream + 0x632BE59BD9B4E019ull) + (i + 1) * 0x9E3779B97F4A7C15ull);
}
__device__ __forceinline__ uint16_t synth_scale(uint64_t bits) {
    const float u = (float)(uint32_t)(bits & 0xffffffu) * (1.0f / 16777216.0f);
    const float v = __fadd_rn(1e-4f, __fmul_rn(u, 9e-4f));
    return __half_as_ushort(__float2half_rn(v));
}

// Block g of the synthetic matrix (stream `stream`) written to blk.
__device__ void synth_q4k_block(uint8_t* blk, uint64_t g, uint64_t seed, uint64_t stream) {
    const uint64_t i0 = g * 32;
    const uint64_t r0 = rand64(seed, stream, i0);
    const uint16_t d = synth_scale(r0), dm = synth_scale(r0 >> 24);
    const uint64_t r1 = rand64(seed, stream, i0 + 1), r2 = rand64(seed, stream, i0 + 2);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; j++) { sc[j] = (r1 >> (6 * j)) & 63; mn[j] = (r2 >> (6 * j)) & 63; }
    uint32_t hdr[4];
    hdr[0] = (uint32_t)d | ((uint32_t)dm << 16);
    uint8_t s[12];
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
    for (int w = 0; w < 3; w++)
        hdr[1 + w] = s[4 * w] | (s[4 * w + 1] << 8) | (s[4 * w + 2] << 16) | ((uint32_t)s[4 * w + 3] << 24);
    uint4* dst = reinterpret_cast<uint4*>(blk);   // 144-byte blocks: 16-byte aligned
    dst[0] = make_uint4(hdr[0], hdr[1], hdr[2], hdr[3]);
    for (int w = 0; w < 8; w++) {
        const uint64_t a = rand64(seed, stream, i0 + 3 + 2 * w), c = rand64(seed, stream, i0 + 4 + 2 * w);
        dst[1 + w] = make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)c, (uint32_t)(c >> 32));
    }
}

__device__ void synth_q6k_block(uint8_t* blk, uint64_t g, uint64_t seed, uint64_t stream) {
    uint16_t* d16 = reinterpret_cast<uint16_t*>(blk);   // 2-byte aligned: write 16-bit halves
    const uint64_t i0 = g * 32;
    for (int w = 0; w < 24; w++) {
        const uint64_t r = rand64(seed, stream, i0 + w);
        for (int k = 0; k < 4; k++) d16[4 * w + k] = (uint16_t)(r >> (16 * k));
    }
    const uint64_t r1 = rand64(seed, stream, i0 + 24), r2 = rand64(seed, stream, i0 + 25);
    uint8_t sc[16];
    for (int j = 0; j < 16; j++) {
        const uint64_t r = j < 8 ? r1 : r2;
        sc[j] = (uint8_t)(int8_t)((int)((r >> (6 * (j & 7))) & 63) - 32);
    }
    for (int j = 0; j < 8; j++) d16[96 + j] = (uint16_t)(sc[2 * j] | (sc[2 * j + 1] << 8));
    d16[104] = synth_scale(rand64(seed, stream, i0 + 26));
}

__device__ void synth_q8_0_block(uint8_t* blk, uint64_t g, uint64_t seed, uint64_t stream) {
    uint16_t* d16 = reinterpret_cast<uint16_t*>(blk);
    const uint64_t i0 = g * 8;
    d16[0] = synth_scale(rand64(seed, stream, i0));
    for (int w = 0; w < 4; w++) {
        const uint64_t r = rand64(seed, stream, i0 + 1 + w);
        for (int k = 0; k < 4; k++) d16[1 + 4 * w + k] = (uint16_t)(r >> (16 * k));
    }
}

// Q5_K: the Q4_K header and nibbles (same words), then 32 bytes of fifth bits.
__device__ void synth_q5k_block(uint8_t* blk, uint64_t g, uint64_t seed, uint64_t stream) {
    alignas(16) uint8_t tmp[GB_Q4K_BYTES];   // synth_q4k_block stores 16-byte words
    synth_q4k_block(tmp, g, seed, stream);   // header words 0-2, nibbles 3-18
    uint4* dst = reinterpret_cast<uint4*>(blk);   // 176-byte blocks: 16-byte aligned
    const uint4* src = reinterpret_cast<const uint4*>(tmp);
    dst[0] = src[0];
    const uint64_t i0 = g * 32;
    for (int w = 0; w < 2; w++) {
        const uint64_t a = rand64(seed, stream, i0 + 19 + 2 * w), c = rand64(seed, stream, i0 + 20 + 2 * w);
        dst[1 + w] = make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)c, (uint32_t)(c >> 32));
    }
    for (int w = 0; w < 8; w++) dst[3 + w] = src[1 + w];
}

// F16 "block" g: 32 halves, each the Irwin-Hall value of k_synth_normal at
// index 32 g + e times 2^-5, rounded to nearest even.
__device__ void synth_f16_block(uint8_t* blk, uint64_t g, uint64_t seed, uint64_t stream) {
    uint16_t* h = reinterpret_cast<uint16_t*>(blk);
    for (int e = 0; e < 32; e++) {
        const uint64_t i = g * 32 + e;
        int32_t acc = 0;
        for (int w = 0; w < 3; w++) {
            const uint64_t r = rand64(seed, stream, 3 * i + w);
            acc += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) + (int32_t)((r >> 32) & 0xffff) +
                   (int32_t)((r >> 48) & 0xffff);
        }
        h[e] = __half_as_ushort(__float2half_rn((float)(acc + 6 - 393216) * (1.0f / 2097152.0f)));
    }
}

// Local block b = r * sn + j (r < rows, j < sn) is global block
// (row0 + r) * nbg + c0 + j, written at output block r * ldo + j: a row or
// column slice of a larger synthetic matrix (tensor-parallel shards) gets
// exactly the bytes of the full matrix.  The identity map is rows = 1,
// sn = ldo = nbg = n, row0 = c0 = 0.
struct SynthMap {
    uint64_t row0, nbg, c0, sn, ldo;
};
template <int DT>
__global__ void k_synth_map(uint8_t* B, uint64_t n_local, uint64_t seed, uint64_t stream, SynthMap m) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_local) return;
    const uint64_t r = b / m.sn, j = b - r * m.sn;
    const uint64_t g = (m.row0 + r) * m.nbg + m.c0 + j;
    constexpr int BYTES = DT == GB_DT_Q4_K ? GB_Q4K_BYTES : DT == GB_DT_Q6_K ? GB_Q6K_BYTES
                        : DT == GB_DT_Q5_K ? GB_Q5K_BYTES : DT == GB_DT_F16 ? GB_F16_BYTES : GB_Q80_BYTES;
    uint8_t* blk = B + (r * m.ldo + j) * BYTES;
    if (DT == GB_DT_Q4_K) synth_q4k_block(blk, g, seed, stream);
    else if (DT == GB_DT_Q6_K) synth_q6k_block(blk, g, seed, stream);
    else if (DT == GB_DT_Q5_K) synth_q5k_block(blk, g, seed, stream);
    else if (DT == GB_DT_F16) synth_f16_block(blk, g, seed, stream);
    else synth_q8_0_block(blk, g, seed, stream);
}

__global__ void k_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        int32_t acc = 0;
        for (int w = 0; w < 3; w++) {
            const uint64_t r = rand64(seed, stream, 3 * (uint64_t)i + w);
            acc += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) +
                   (int32_t)((r >> 32) & 0xffff) + (int32_t)((r >> 48) & 0xffff);
        }
        out[i] = (float)(acc + 6 - 393216) * (1.0f / 65536.0f);
    }
}

__global__ void k_fill(float* out, size_t n, float v) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

}  // namespace gb

// ======================================================================= C ABI
using namespace gb;

extern "C" int gb_dequant(int dtype, const void* blocks, size_t nblocks, float* out, void* stream) {
    if (!blocks || !out) return GB_EINVAL;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (nblocks == 0) return GB_OK;
    const uint8_t* B = static_cast<const uint8_t*>(blocks);
    switch (dtype) {
        case GB_DT_Q4_K: k_dequant_q4k<<<(unsigned)((nblocks * 128 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_Q6_K: k_dequant_q6k<<<(unsigned)((nblocks * 64 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_Q8_0: k_dequant_q8_0<<<(unsigned)((nblocks * 32 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_Q5_K: k_dequant_q5k<<<(unsigned)((nblocks * 128 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_F16:
            if (reinterpret_cast<uintptr_t>(blocks) & 1) return GB_EINVAL;
            k_dequant_f16<<<(unsigned)((nblocks * 32 + 255) / 256), 256, 0, st>>>(
                reinterpret_cast<const uint16_t*>(B), nblocks * 32, out);
            break;
        default: return GB_EINVAL;
    }
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

namespace gb {
int synth_blocks_shard(int dtype, void* out, size_t rows, size_t sn, size_t ldo, uint64_t row0, uint64_t nbg,
                       uint64_t c0, uint64_t seed, uint64_t stream_id, cudaStream_t st) {
    if (!out || sn > ldo) return GB_EINVAL;
    const uint64_t n = (uint64_t)rows * sn;
    if (n == 0) return GB_OK;
    const unsigned grid = (unsigned)((n + 255) / 256);
    uint8_t* B = static_cast<uint8_t*>(out);
    const SynthMap m{row0, nbg, c0, sn, ldo};
    switch (dtype) {
        case GB_DT_Q4_K:
            if (reinterpret_cast<uintptr_t>(out) & 15) return GB_EINVAL;
            k_synth_map<GB_DT_Q4_K><<<grid, 256, 0, st>>>(B, n, seed, stream_id, m); break;
        case GB_DT_Q6_K:
            if (reinterpret_cast<uintptr_t>(out) & 1) return GB_EINVAL;
            k_synth_map<GB_DT_Q6_K><<<grid, 256, 0, st>>>(B, n, seed, stream_id, m); break;
        case GB_DT_Q8_0:
            if (reinterpret_cast<uintptr_t>(out) & 1) return GB_EINVAL;
            k_synth_map<GB_DT_Q8_0><<<grid, 256, 0, st>>>(B, n, seed, stream_id, m); break;
        case GB_DT_Q5_K:
            if (reinterpret_cast<uintptr_t>(out) & 15) return GB_EINVAL;
            k_synth_map<GB_DT_Q5_K><<<grid, 256, 0, st>>>(B, n, seed, stream_id, m); break;
        case GB_DT_F16:
            if (reinterpret_cast<uintptr_t>(out) & 1) return GB_EINVAL;
            k_synth_map<GB_DT_F16><<<grid, 256, 0, st>>>(B, n, seed, stream_id, m); break;
        default: return GB_EINVAL;
    }
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
}  // namespace gb

extern "C" int gb_synth_blocks(int dtype, void* blocks, size_t nblocks, uint64_t seed, uint64_t stream_id,
                               void* stream) {
    if (!blocks) return GB_EINVAL;
    return gb::synth_blocks_shard(dtype, blocks, 1, nblocks, nblocks, 0, nblocks, 0, seed, stream_id,
                                  static_cast<cudaStream_t>(stream));
}

extern "C" int gb_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream_id, void* stream) {
    if (!out) return GB_EINVAL;
    if (n == 0) return GB_OK;
    const size_t g = (n + 255) / 256;
    k_synth_normal<<<(unsigned)(g < 4096 ? g : 4096), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, stream_id);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

extern "C" int gb_fill_f32(float* out, size_t n, float v, void* stream) {
    if (!out) return GB_EINVAL;
    if (n == 0) return GB_OK;
    const size_t g = (n + 255) / 256;
    k_fill<<<(unsigned)(g < 4096 ? g : 4096), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, n, v);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
