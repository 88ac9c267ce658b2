// gb_gemm.cu -- prefill GEMM on the sm_100a tensor cores (tcgen05):
//     Y[t][n] = sum_k X[t][k] W[n][k]  (+ R[t][n])
// for T prompt tokens at once, with W in GGUF Q4_K / Q6_K / Q8_0 blocks
// (dequantised on the fly) or plain fp32.  This is the T > 1 half of the
// reference's linear_dispatch (src/engine/engine.c:87-154), which loops the
// matvec once per token; the reference's GPU prefill hook is a stub
// (src/engine/gpu_prefill.c:3-20).
//
// Precision: fp32-equivalent ("3xTF32").  Every weight is dequantised to its
// fp32 value (the reference's per-weight formula), every activation is fp32;
// both are split into a tf32 part and an fp32 remainder (x = hi + lo), and
// the tensor cores accumulate hi.hi + hi.lo + lo.hi in fp32 tensor memory --
// about 22 bits of each operand, so a prompt pass agrees with the reference's
// fp32 arithmetic as closely as the decode matvecs do.
//
// CTA tile: 128 weight rows (the MMA's M) x BT = 128 tokens (its N), K in
// chunks of 32.  Warps 0-3 convert: thread r dequantises row r's 32 weights
// of the chunk and splits token r's 32 activations, storing both into a
// 3-stage shared-memory ring in the tensor cores' K-major layout (gb_tc.cuh).
// Warp 4 allocates the tensor memory and one of its lanes issues the 12 MMAs
// of a chunk (4 k-steps x 3 products), then commits them to the stage's
// "empty" barrier so the converters may refill it.  The tensor cores' fp32
// accumulation is not round-to-nearest, so its error grows with the number
// of MMAs summed into one accumulator: every 256 columns of K the MMAs start
// a fresh accumulator (two in tensor memory, alternating), and warps 5-12
// read each finished one back and add it into fp32 registers (lane r = weight
// row, 64 of the 128 token columns per warp), then write Y after the last.
// Every wait is bounded (2 s of %globaltimer) and records GB_ETIMEOUT in the
// caller's error word (gb_gemm: a module-wide word read by gb_gemm_error).
#include "gb_common.cuh"
#include "gb_internal.h"
#include "gb_mt.cuh"
#include "gb_tc.cuh"

namespace gb {

constexpr int GM_ROWS = 128;             // weight rows per CTA (MMA M)
constexpr int GM_BT = 128;               // tokens per CTA (MMA N)
constexpr int GM_BK = 32;                // K per stage
constexpr int GM_S = 3;                  // ring stages
constexpr int GM_KG = 8;                 // stages summed into one accumulator (256 columns of K)
constexpr int GM_TILE_A = GM_ROWS * GM_BK * 4;   // 16 KB (one of hi / lo)
constexpr int GM_TILE_B = GM_BT * GM_BK * 4;     // 16 KB
constexpr int GM_STAGE = 2 * GM_TILE_A + 2 * GM_TILE_B;
constexpr int GM_READERS = 8;            // accumulator-reader warps (5 .. 12)
constexpr int GM_THREADS = (5 + GM_READERS) * 32;
constexpr int GM_SMEM = GM_S * GM_STAGE + 1024;
constexpr uint32_t GM_TMEM_COLS = 2 * GM_BT;   // two accumulators

__device__ unsigned g_gemm_err;

// Row r's 32 weights k0 .. k0 + 31 as fp32 values (the reference's formulas).
template <int DT>
__device__ __forceinline__ void dequant32(const uint8_t* __restrict__ W, int n, int K, int k0, float (&w)[32]) {
    if constexpr (DT == GB_DT_F32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(W) + (size_t)n * K + k0);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldg(p + i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    } else if constexpr (DT == GB_DT_Q8_0) {
        // quant_matvec_q8_0.c:41-78: w = q * d (block of 32)
        const uint8_t* blk = W + ((size_t)n * (K / 32) + k0 / 32) * GB_Q80_BYTES;
        const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
#pragma unroll
        for (int i = 0; i < 32; i++) w[i] = (float)(int8_t)blk[2 + i] * d;
    } else if constexpr (DT == GB_DT_Q4_K) {
        // quant_matvec_q4_k.c:95-126: d1 = d sc, m1 = dmin m, w = d1 q - m1 (one rounding)
        const int nb = K / 256, b = k0 >> 8, j = (k0 >> 5) & 7;
        const uint8_t* blk = W + ((size_t)n * nb + b) * GB_Q4K_BYTES;
        const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
        const float dmin = f16_bits_to_f32(blk[2] | (blk[3] << 8));
        const uint8_t* s = blk + 4;
        uint32_t sc, mn;
        if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
        else { sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
        const float d1 = d * (float)sc, m1 = dmin * (float)mn;
        const uint8_t* q = blk + 16 + 32 * (j >> 1);
        const int sh = (j & 1) * 4;
#pragma unroll
        for (int i = 0; i < 32; i++) w[i] = fmaf(d1, (float)((q[i] >> sh) & 0xF), -m1);
    } else {
        // quant_matvec_q6_k.c:75-92: w = d sc (q - 32), q = ql nibble | qh bits << 4
        const int nb = K / 256, b = k0 >> 8, kl = k0 & 255, h = kl >> 7, G = (kl >> 5) & 3;
        const uint8_t* blk = W + ((size_t)n * nb + b) * GB_Q6K_BYTES;
        const uint8_t* ql = blk + 64 * h + ((G & 1) ? 32 : 0);
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192) + 8 * h + 2 * G;
        const float d = f16_bits_to_f32(blk[208] | (blk[209] << 8));
        const float ds0 = d * (float)sc[0], ds1 = d * (float)sc[1];
        const int nsh = (G >> 1) * 4, hsh = 2 * G;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int q = ((ql[i] >> nsh) & 0xF) | (((qh[i] >> hsh) & 3) << 4);
            w[i] = (i < 16 ? ds0 : ds1) * (float)(q - 32);
        }
    }
}

__device__ __forceinline__ bool gm_wait(uint32_t bar, uint32_t parity, unsigned* err) {
    if (mbs_test(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbs_test(bar, parity))
        if (gtimer() - t0 > MT_WAIT_NS) {
            atomicExch(err ? err : &g_gemm_err, (unsigned)(-GB_ETIMEOUT));
            return false;
        }
    return true;
}

// Store 32 fp32 values of one row, split into tf32 hi / lo, into the two
// K-major tiles of R rows.
template <int R>
__device__ __forceinline__ void store_split(uint8_t* hi, uint8_t* lo, int r, const float (&v)[32]) {
#pragma unroll
    for (int g = 0; g < 8; g++) {
        float h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; e++) tc::split_tf32(v[4 * g + e], h[e], l[e]);
        const uint32_t off = tc::tile_off(r, 4 * g, R);
        *reinterpret_cast<float4*>(hi + off) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(lo + off) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

template <int DT>
__global__ void __launch_bounds__(GM_THREADS, 1)
k_gemm(const uint8_t* __restrict__ W, const float* __restrict__ X, float* Y, const float* R, int N, int K, int T,
       unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned stage ring; barriers and the tensor-memory address
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[2 * GM_S + 4];
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * GM_ROWS, t0 = blockIdx.y * GM_BT;
    const uint32_t full = tc::smem_u32(&bars[0]), empty = full + 8 * GM_S;
    const uint32_t accfull = full + 16 * GM_S, accfree = accfull + 16;   // [2] each
    const int nk = K / GM_BK;
    const int ng = (nk + GM_KG - 1) / GM_KG;   // accumulator groups
    if (threadIdx.x == 0) {
        for (int s = 0; s < GM_S; s++) {
            mbs_init(full + 8 * s, 4);   // one arrival per converter warp
            mbs_init(empty + 8 * s, 1);  // the MMA commit
        }
        for (int a = 0; a < 2; a++) {
            mbs_init(accfull + 8 * a, 1);            // the MMA commit of a group
            mbs_init(accfree + 8 * a, GM_READERS);   // every reader warp has taken it
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) tc::tmem_alloc(&tmem_slot, GM_TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;

    if (warp == 4) {   // ---- MMA issue (one lane)
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_tf32(GM_ROWS, GM_BT);
            constexpr uint32_t LBO_A = GM_ROWS / 8 * 128, LBO_B = GM_BT / 8 * 128;
            bool ok = true;
            for (int g = 0; g < ng && ok; g++) {
                const int a = g & 1;
                if (g >= 2) ok = gm_wait(accfree + 8 * a, ((g >> 1) - 1) & 1, err);
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t acc = tmem + (uint32_t)(a * GM_BT);
                const int k1 = min(nk, (g + 1) * GM_KG);
                for (int kc = g * GM_KG; kc < k1; kc++) {
                    const int s = kc % GM_S;
                    ok = gm_wait(full + 8 * s, (kc / GM_S) & 1, err);
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t base = tc::smem_u32(smem + (size_t)s * GM_STAGE);
                    const uint32_t ahi = base, alo = base + GM_TILE_A, bhi = base + 2 * GM_TILE_A,
                                   blo = bhi + GM_TILE_B;
#pragma unroll
                    for (int ks = 0; ks < GM_BK / 8; ks++) {
                        const uint64_t dah = tc::smem_desc(ahi + ks * 2 * LBO_A, LBO_A, 128);
                        const uint64_t dal = tc::smem_desc(alo + ks * 2 * LBO_A, LBO_A, 128);
                        const uint64_t dbh = tc::smem_desc(bhi + ks * 2 * LBO_B, LBO_B, 128);
                        const uint64_t dbl = tc::smem_desc(blo + ks * 2 * LBO_B, LBO_B, 128);
                        tc::mma_tf32(acc, dah, dbh, idesc, kc > g * GM_KG || ks > 0);
                        tc::mma_tf32(acc, dah, dbl, idesc, true);
                        tc::mma_tf32(acc, dal, dbh, idesc, true);
                    }
                    tc::mma_commit(empty + 8 * s);   // the stage may be refilled once these MMAs are done
                }
                tc::mma_commit(accfull + 8 * a);     // the group's partial sum is complete
            }
        }
        __syncwarp();
    } else if (warp < 4) {   // ---- warps 0-3: convert
        const int r = threadIdx.x;   // weight row n0 + r and token t0 + r of every chunk
        const int n = n0 + r, t = t0 + r;
        bool ok = true;
        for (int kc = 0; kc < nk; kc++) {
            const int s = kc % GM_S;
            if (kc >= GM_S && ok) ok = gm_wait(empty + 8 * s, ((kc / GM_S) - 1) & 1, err);
            uint8_t* st = smem + (size_t)s * GM_STAGE;
            float v[32];
            if (n < N) {
                dequant32<DT>(W, n, K, kc * GM_BK, v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            store_split<GM_ROWS>(st, st + GM_TILE_A, r, v);
            if (t < T) {
                const float4* p = reinterpret_cast<const float4*>(X + (size_t)t * K + kc * GM_BK);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float4 u = __ldg(p + i);
                    v[4 * i] = u.x; v[4 * i + 1] = u.y; v[4 * i + 2] = u.z; v[4 * i + 3] = u.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            store_split<GM_BT>(st + 2 * GM_TILE_A, st + 2 * GM_TILE_A + GM_TILE_B, r, v);
            tc::fence_async_smem();   // generic-proxy stores -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbs_arrive(full + 8 * s);
        }
    } else {   // ---- warps 5-12: sum the accumulators in fp32, then write Y
        const int q = warp & 3;                       // tensor-memory lane quarter this warp may read
        const int c0 = (warp - 5) >= 4 ? GM_BT / 2 : 0;   // the warp's half of the token columns
        const int r = q * 32 + lane, n = n0 + r;
        float sum[GM_BT / 2];
#pragma unroll
        for (int i = 0; i < GM_BT / 2; i++) sum[i] = 0.f;
        bool ok = true;
        for (int g = 0; g < ng && ok; g++) {
            const int a = g & 1;
            ok = gm_wait(accfull + 8 * a, (g >> 1) & 1, err);
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * GM_BT + c0);
#pragma unroll
            for (int c = 0; c < GM_BT / 2; c += 16) {
                float v[16];
                tc::tmem_ld16(base + c, v);
#pragma unroll
                for (int i = 0; i < 16; i++) sum[c + i] += v[i];
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbs_arrive(accfree + 8 * a);
        }
        if (ok && n < N) {
#pragma unroll
            for (int i = 0; i < GM_BT / 2; i++) {
                const int tt = t0 + c0 + i;
                if (tt < T) {
                    const size_t o = (size_t)tt * N + n;
                    Y[o] = sum[i] + (R ? R[o] : 0.f);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 4) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, GM_TMEM_COLS);
    }
}

template <int DT>
static int launch_gemm(const void* W, const float* X, float* Y, const float* R, int N, int K, int T, cudaStream_t st,
                       unsigned* err) {
    GB_CUDA_TRY(set_smem_once(reinterpret_cast<const void*>(k_gemm<DT>), GM_SMEM));
    dim3 grid((N + GM_ROWS - 1) / GM_ROWS, (T + GM_BT - 1) / GM_BT);
    k_gemm<DT><<<grid, GM_THREADS, GM_SMEM, st>>>(static_cast<const uint8_t*>(W), X, Y, R, N, K, T, err);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

int gemm_launch(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T,
                cudaStream_t st, unsigned* err) {
    if (!W || !X || !Y || N <= 0 || K <= 0 || T <= 0) return GB_EINVAL;
    if ((reinterpret_cast<uintptr_t>(X) & 15) || (dtype == GB_DT_F32 && (reinterpret_cast<uintptr_t>(W) & 15)))
        return GB_EINVAL;
    switch (dtype) {
        case GB_DT_F32: return K % GM_BK ? GB_ESHAPE : launch_gemm<GB_DT_F32>(W, X, Y, R, N, K, T, st, err);
        case GB_DT_Q8_0: return K % 32 ? GB_ESHAPE : launch_gemm<GB_DT_Q8_0>(W, X, Y, R, N, K, T, st, err);
        case GB_DT_Q4_K: return K % 256 ? GB_ESHAPE : launch_gemm<GB_DT_Q4_K>(W, X, Y, R, N, K, T, st, err);
        case GB_DT_Q6_K: return K % 256 ? GB_ESHAPE : launch_gemm<GB_DT_Q6_K>(W, X, Y, R, N, K, T, st, err);
        default: return GB_EINVAL;
    }
}

}  // namespace gb

extern "C" int gb_gemm(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T,
                       void* stream) {
    return gb::gemm_launch(dtype, W, X, Y, R, N, K, T, static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int gb_gemm_error(int clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, gb::g_gemm_err, sizeof(v)) != cudaSuccess) return GB_ECUDA;
    if (clear && v) {
        const unsigned z = 0;
        if (cudaMemcpyToSymbol(gb::g_gemm_err, &z, sizeof(z)) != cudaSuccess) return GB_ECUDA;
    }
    return -(int)v;
}
