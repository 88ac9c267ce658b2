// gb_gemm.cu -- prefill GEMM on the sm_100a tensor cores (tcgen05):
//     Y[t][n] = sum_k X[t][k] W[n][k]  (+ R[t][n])
// for T prompt tokens at once, with W in GGUF Q4_K / Q6_K / Q8_0 / Q5_K blocks
// (dequantised on the fly) or plain fp32 / fp16 rows.  This is the T > 1 half of the
// reference's linear_dispatch (src/engine/engine.c:87-154), which loops the
// matvec once per token; the reference's GPU prefill hook is a stub
// (src/engine/gpu_prefill.c:3-20).
//
// Precision: fp32-equivalent.  Every weight is dequantised to its fp32 value
// (the reference's per-weight formula), every activation is fp32; both are
// split into an 11-significant-bit part and the remainder (x = hi + lo), and
// the tensor cores accumulate hi.hi + hi.lo + lo.hi in fp32 tensor memory --
// about 22 bits of each operand, so a prompt pass agrees with the reference's
// fp32 arithmetic as closely as the decode matvecs do.  The operands are fp16
// pairs by default ("3xF16", kind::f16: twice the tensor rate of tf32 and
// half the shared-memory bytes); fp16's narrow exponent range is handled by
// powers of two -- each weight row by 2^e_n chosen from its blocks' scale
// fields (an upper bound of |w|), each token row of X by 2^e_t chosen from
// its largest |x| (gemm_row_absmax), both to below 2^15 -- taken back out
// exactly when Y is written.  GB_GEMM_KIND=tf32 selects tf32 pairs ("3xTF32",
// no scaling) instead.
//
// CTA tile: 128 weight rows (the MMA's M) x BT = 128 or 256 tokens (its N;
// 256 when that grid still fills every SM), K in chunks of 32 through a
// shared-memory ring in the tensor cores' K-major layout (gb_tc.cuh): 6 / 4
// stages of fp16 pairs at BT 128 / 256 (3 / 2 of tf32 pairs).  Warps 0-3 convert weights: thread r dequantises row
// r's 32 weights of the chunk (Q4_K / Q5_K: 16-byte loads of a chunk pair's
// bytes, three / two pairs in flight; Q6_K: 4-byte words of a 128-column
// half-block, the next one loaded before this one is converted).  Warp 13
// loads each chunk's raw activation tile [BT tokens][32] fp32 by TMA into the
// stage, and warps 9-12 split it in place.  Warp 4 allocates the tensor
// memory and one of its lanes issues the MMAs of a chunk (2 k-steps of 16
// for fp16, 4 of 8 for tf32, x 3 products), then commits them to the stage's "empty" barrier so the
// converters may refill it.  The tensor cores' fp32 accumulation is not
// round-to-nearest, so its error grows with the number of MMAs summed into
// one accumulator: every 256 columns of K (512 at BT 256) the MMAs start a
// fresh accumulator (two in tensor memory, alternating; one at BT 256,
// refilled once read), and
// warps 5-8 read each finished one back and add it to a running fp32 sum kept
// in a further tensor-memory region (lane r = weight row), then write Y after
// the last.
// Every wait is bounded (2 s of %globaltimer) and records GB_ETIMEOUT in the
// caller's error word (gb_gemm: a module-wide word read by gb_gemm_error).
#include "gb_common.cuh"
#include "gb_internal.h"
#include "gb_mt.cuh"
#include "gb_tc.cuh"

#include <string.h>

namespace gb {

constexpr int GM_ROWS = 128;             // weight rows per CTA (MMA M)
constexpr int GM_BK = 32;                // K per stage
constexpr int GM_READERS = 4;            // accumulator-reader warps (5 .. 8)
constexpr int GM_XWARPS = 4;             // activation converter warps (9 .. 12)
constexpr int GM_XPROD = 5 + GM_READERS + GM_XWARPS;   // warp 13: activation tile loads (TMA)
constexpr int GM_THREADS = (GM_XPROD + 1) * 32;

// Token-tile size BT (the MMA's N): 128 (two accumulators alternating) or
// 256 (one accumulator, refilled once the readers have taken it); operands
// as fp16 (H16) or tf32 pairs.  A stage holds the hi and lo tiles of A (the
// weights) and B (the activations); the raw fp32 activation tile lands in
// B's hi (and, for fp16, lo) tile and is split in place.
template <int BT, bool H16>
struct GmCfg {
    static constexpr int EB = H16 ? 2 : 4;                     // operand element bytes
    static constexpr int TILE_A = GM_ROWS * GM_BK * EB;        // one of hi / lo: 8 / 16 KB
    static constexpr int TILE_B = BT * GM_BK * EB;
    static constexpr int XRAW = BT * GM_BK * 4;                // the raw fp32 activation tile
    static constexpr int STAGE = 2 * TILE_A + 2 * TILE_B;
    static constexpr int S = H16 ? (BT == 256 ? 4 : 6) : (BT == 256 ? 2 : 3);   // ring stages
    static constexpr int NACC = BT == 256 ? 1 : 2;              // accumulators in tensor memory
    // chunks per accumulator group: 512 / 256 columns of K for tf32, twice
    // that for fp16 (the same 192 / 96 MMAs per accumulator)
    static constexpr int KG = (BT == 256 ? 16 : 8) * (H16 ? 2 : 1);
    static constexpr int SMEM = S * STAGE + 1024;
    static constexpr uint32_t TMEM_COLS = 512;                  // NACC x BT accumulator + BT running sum
    static_assert(XRAW <= 2 * TILE_B, "the raw activation tile fits B's tiles");
};
static_assert(GmCfg<256, false>::SMEM <= 227 * 1024 && GmCfg<128, false>::SMEM <= 227 * 1024, "shared memory");
static_assert(GmCfg<256, true>::SMEM <= 227 * 1024 && GmCfg<128, true>::SMEM <= 227 * 1024, "shared memory");

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
    } else if constexpr (DT == GB_DT_F16) {   // exact half -> float
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(W) + (size_t)n * K + k0);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 v = __ldg(p + i);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[e]));
                w[8 * i + 2 * e] = f.x;
                w[8 * i + 2 * e + 1] = f.y;
            }
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

// The same for fp16 pairs (values already scaled below 2^15).
template <int R>
__device__ __forceinline__ void store_split16(uint8_t* hi, uint8_t* lo, int r, const float (&v)[32]) {
#pragma unroll
    for (int g = 0; g < 4; g++) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; e++) tc::split_f16x2(v[8 * g + 2 * e], v[8 * g + 2 * e + 1], h[e], l[e]);
        const uint32_t off = tc::tile_off16(r, 8 * g, R);
        *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// Scale exponent of weight row n for fp16 operands, from an upper bound of
// its |w|: per block |d| * max|sc * q| + |dmin| * max(m) (Q4_K 15 * 63 and
// 63, Q5_K 31 * 63 and 63), |d| * 128 * 32 (Q6_K), |d| * 128 (Q8_0), the
// row's largest |w| (F32); fp16 rows are exact as they are (0).
template <int DT>
__device__ int row_scale_exp(const uint8_t* __restrict__ W, int n, int K) {
    float b = 0.f;
    if constexpr (DT == GB_DT_F16) {
        return 0;
    } else if constexpr (DT == GB_DT_F32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(W) + (size_t)n * K);
#pragma unroll 8
        for (int i = 0; i < K / 4; i++) {
            const float4 v = __ldg(p + i);
            b = fmaxf(b, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else if constexpr (DT == GB_DT_Q4_K || DT == GB_DT_Q5_K) {
        constexpr int BB = DT == GB_DT_Q5_K ? GB_Q5K_BYTES : GB_Q4K_BYTES;
        constexpr float QM = DT == GB_DT_Q5_K ? 31.f * 63.f : 15.f * 63.f;
        const int nb = K / 256;
        const uint8_t* row = W + (size_t)n * nb * BB;
#pragma unroll 8
        for (int i = 0; i < nb; i++) {
            const uint32_t h = __ldg(reinterpret_cast<const uint32_t*>(row + (size_t)i * BB));
            b = fmaxf(b, fabsf(f16_bits_to_f32(h & 0xFFFF)) * QM + fabsf(f16_bits_to_f32(h >> 16)) * 63.f);
        }
    } else if constexpr (DT == GB_DT_Q6_K) {
        const int nb = K / 256;
        const uint8_t* row = W + (size_t)n * nb * GB_Q6K_BYTES;
#pragma unroll 8
        for (int i = 0; i < nb; i++)
            b = fmaxf(b, fabsf(f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(row + (size_t)i * GB_Q6K_BYTES + 208)))) *
                             4096.f);
    } else {   // Q8_0
        const int nb = K / 32;
        const uint8_t* row = W + (size_t)n * nb * GB_Q80_BYTES;
#pragma unroll 8
        for (int i = 0; i < nb; i++)
            b = fmaxf(b, fabsf(f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(row + (size_t)i * GB_Q80_BYTES)))) *
                             128.f);
    }
    return tc::f16_scale_exp(__float_as_uint(b));
}

// SW (SwiGLU): W holds the gate rows and W2 the up rows of an FFN; a CTA
// takes 64 gate rows and the same 64 up rows (its 128 weight rows), and the
// readers write Y[t][f] = silu(gate) * up (k_silu_mul's rounding) for its 64
// columns instead of the two products.
// H16: fp16 operand pairs; the activations come split (gemm_split_x): xmap
// and xlmap view their hi and lo halves, and xinv holds the token scales'
// inverses.  Else tf32 pairs: xmap views the fp32 X, which warps 9-12 split
// in shared memory (xlmap and xinv unused).
template <int DT, int BT, bool SW, bool H16>
__global__ void __launch_bounds__(GM_THREADS, 1)
k_gemm(const __grid_constant__ CUtensorMap xmap, const uint8_t* __restrict__ W, const uint8_t* __restrict__ W2, float* Y,
       const float* R, const __grid_constant__ CUtensorMap xlmap, const float* __restrict__ xinv, int N, int ldy, int K,
       int T, unsigned* err) {
    using C = GmCfg<BT, H16>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned stage ring; barriers and the tensor-memory address
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[3 * C::S + 4];
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * (SW ? GM_ROWS / 2 : GM_ROWS), t0 = blockIdx.y * BT;
    const uint32_t full = tc::smem_u32(&bars[0]), empty = full + 8 * C::S, xfull = full + 16 * C::S;
    const uint32_t accfull = full + 24 * C::S, accfree = accfull + 16;   // [2] each
    const int nk = K / GM_BK;
    const int ng = (nk + C::KG - 1) / C::KG;   // accumulator groups
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; s++) {
            // one arrival per converter warp (W, and for tf32 X), or for
            // fp16 the W converters and the activation loads' expect_tx
            mbs_init(full + 8 * s, H16 ? 4 + 1 : 4 + GM_XWARPS);
            mbs_init(empty + 8 * s, 1);  // the MMA commit
            mbs_init(xfull + 8 * s, 1);  // the activation tile's TMA load
        }
        for (int a = 0; a < 2; a++) {
            mbs_init(accfull + 8 * a, 1);            // the MMA commit of a group
            mbs_init(accfree + 8 * a, GM_READERS);   // every reader warp has taken it
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) tc::tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;

    if (warp == 4) {   // ---- MMA issue (one lane)
        if (lane == 0) {
            constexpr uint32_t idesc = H16 ? tc::idesc_f16(GM_ROWS, BT) : tc::idesc_tf32(GM_ROWS, BT);
            constexpr int KS = H16 ? 16 : 8;   // K per MMA
            constexpr uint32_t LBO_A = GM_ROWS / 8 * 128, LBO_B = BT / 8 * 128;
            bool ok = true;
            for (int g = 0; g < ng && ok; g++) {
                const int a = g % C::NACC;   // accumulator of group g; reused once the readers took group g - NACC
                if (g >= C::NACC) ok = gm_wait(accfree + 8 * a, ((g / C::NACC) - 1) & 1, err);
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t acc = tmem + (uint32_t)(a * BT);
                const int k1 = min(nk, (g + 1) * C::KG);
                for (int kc = g * C::KG; kc < k1; kc++) {
                    const int s = kc % C::S;
                    ok = gm_wait(full + 8 * s, (kc / C::S) & 1, err);
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t base = tc::smem_u32(smem + (size_t)s * C::STAGE);
                    const uint32_t ahi = base, alo = base + C::TILE_A, bhi = base + 2 * C::TILE_A,
                                   blo = bhi + C::TILE_B;
#pragma unroll
                    for (int ks = 0; ks < GM_BK / KS; ks++) {   // each k-step spans two core-matrix column groups
                        const uint64_t dah = tc::smem_desc(ahi + ks * 2 * LBO_A, LBO_A, 128);
                        const uint64_t dal = tc::smem_desc(alo + ks * 2 * LBO_A, LBO_A, 128);
                        const uint64_t dbh = tc::smem_desc(bhi + ks * 2 * LBO_B, LBO_B, 128);
                        const uint64_t dbl = tc::smem_desc(blo + ks * 2 * LBO_B, LBO_B, 128);
                        if constexpr (H16) {
                            tc::mma_f16(acc, dah, dbh, idesc, kc > g * C::KG || ks > 0);
                            tc::mma_f16(acc, dah, dbl, idesc, true);
                            tc::mma_f16(acc, dal, dbh, idesc, true);
                        } else {
                            tc::mma_tf32(acc, dah, dbh, idesc, kc > g * C::KG || ks > 0);
                            tc::mma_tf32(acc, dah, dbl, idesc, true);
                            tc::mma_tf32(acc, dal, dbh, idesc, true);
                        }
                    }
                    tc::mma_commit(empty + 8 * s);   // the stage may be refilled once these MMAs are done
                }
                tc::mma_commit(accfull + 8 * a);     // the group's partial sum is complete
            }
        }
        __syncwarp();
    } else if (warp < 4) {   // ---- warps 0-3: weight rows n0 + threadIdx.x
        const int r = threadIdx.x;
        // SW: rows 0-63 are gate rows n0 .., rows 64-127 the same up rows (W2)
        const int n = SW ? n0 + (r & 63) : n0 + r;
        const uint8_t* Wm = (SW && r >= 64) ? W2 : W;
        // fp16 operands: the row scaled by 2^e (folded into the block scales)
        const float rs = H16 && n < N ? tc::pow2f(row_scale_exp<DT>(Wm, n, K)) : 1.f;
        bool ok = true;
        auto put = [&](int kc, const float (&v)[32]) {   // one chunk into its stage
            const int s = kc % C::S;
            if (kc >= C::S && ok) ok = gm_wait(empty + 8 * s, ((kc / C::S) - 1) & 1, err);
            uint8_t* st = smem + (size_t)s * C::STAGE;
            if constexpr (H16) store_split16<GM_ROWS>(st, st + C::TILE_A, r, v);
            else store_split<GM_ROWS>(st, st + C::TILE_A, r, v);
            tc::fence_async_smem();   // generic-proxy stores -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbs_arrive(full + 8 * s);
        };
        if constexpr (DT == GB_DT_Q4_K || DT == GB_DT_Q5_K) {
            // chunks 2p and 2p + 1 share 32 bytes of nibbles (low / high) and,
            // for Q5_K, the 32 bytes of fifth bits (bit j of byte i for
            // sub-block j); the next pair's bytes are loaded before this pair
            // is converted
            constexpr bool Q5 = DT == GB_DT_Q5_K;
            constexpr int BB = Q5 ? GB_Q5K_BYTES : GB_Q4K_BYTES, QS = Q5 ? 48 : 16;
            const int nb = K / 256;
            const uint8_t* row = Wm + (size_t)(n < N ? n : 0) * nb * BB;
            struct Raw { uint4 hd, qa, qb, ha, hb; };
            auto load = [&](int p, Raw& w) {
                const uint8_t* blk = row + (size_t)(p >> 2) * BB;
                w.hd = __ldg(reinterpret_cast<const uint4*>(blk));   // d, dmin, 12 scale bytes
                w.qa = __ldg(reinterpret_cast<const uint4*>(blk + QS + 32 * (p & 3)));
                w.qb = __ldg(reinterpret_cast<const uint4*>(blk + QS + 16 + 32 * (p & 3)));
                if (Q5) {
                    w.ha = __ldg(reinterpret_cast<const uint4*>(blk + 16));
                    w.hb = __ldg(reinterpret_cast<const uint4*>(blk + 32));
                } else {
                    w.ha = w.hb = make_uint4(0u, 0u, 0u, 0u);
                }
            };
            // D pairs in flight (3 for Q4_K, 2 for Q5_K's larger pairs): the
            // loads of pair p + D are issued before pair p is converted
            constexpr int D = Q5 ? 2 : 3;
            const int np = nk / 2;
            Raw cur, n1, n2;
            load(0, cur);
            n1 = cur;
            n2 = cur;
            if (np > 1) load(1, n1);
            if (D == 3 && np > 2) load(2, n2);
            for (int p = 0; p < np; p++) {
                Raw n3 = D == 3 ? n2 : n1;
                if (p + D < np) load(p + D, n3);
                const uint4 hd = cur.hd;
                const float d = f16_bits_to_f32(hd.x & 0xFFFF), dmin = f16_bits_to_f32(hd.x >> 16);
                const uint32_t sw[3] = {hd.y, hd.z, hd.w};
                const uint32_t qw[8] = {cur.qa.x, cur.qa.y, cur.qa.z, cur.qa.w, cur.qb.x, cur.qb.y, cur.qb.z, cur.qb.w};
                const uint32_t hw[8] = {cur.ha.x, cur.ha.y, cur.ha.z, cur.ha.w, cur.hb.x, cur.hb.y, cur.hb.z, cur.hb.w};
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int j = 2 * (p & 3) + h;   // sub-block of the 256-column block
                    auto sbyte = [&](int i) { return (sw[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
                    uint32_t sc, mn;
                    if (j < 4) { sc = sbyte(j) & 63; mn = sbyte(j + 4) & 63; }
                    else { sc = (sbyte(j + 4) & 0xF) | ((sbyte(j - 4) >> 6) << 4); mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4); }
                    const float d1 = d * (float)sc * rs, m1 = dmin * (float)mn * rs;   // exact: rs is 2^e
                    float v[32];
#pragma unroll
                    for (int wi = 0; wi < 8; wi++) {
                        uint32_t code = (qw[wi] >> (4 * h)) & 0x0F0F0F0Fu;   // 4 codes, one per byte
                        if (Q5) code |= ((hw[wi] >> j) & 0x01010101u) << 4;
                        v[4 * wi + 0] = fmaf(d1, tc::byte_as_float<0>(code, 0.f), -m1);
                        v[4 * wi + 1] = fmaf(d1, tc::byte_as_float<1>(code, 0.f), -m1);
                        v[4 * wi + 2] = fmaf(d1, tc::byte_as_float<2>(code, 0.f), -m1);
                        v[4 * wi + 3] = fmaf(d1, tc::byte_as_float<3>(code, 0.f), -m1);
                    }
                    if (n >= N) {
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = 0.f;
                    }
                    put(2 * p + h, v);
                }
                if (D == 3) {
                    cur = n1;
                    n1 = n2;
                    n2 = n3;
                } else {
                    cur = n1;
                    n1 = n3;
                }
            }
        } else if constexpr (DT == GB_DT_Q6_K) {
            // one 128-column half-block (4 chunks) per step: its ql (64 B),
            // qh (32 B), scales (8 B) and d as 4-byte words from the 2-byte
            // aligned block (realigned by funnel shifts); the next half-block
            // is loaded before this one is converted
            const int nb = K / 256;
            const uint8_t* row = Wm + (size_t)(n < N ? n : 0) * nb * GB_Q6K_BYTES;
            struct Raw { uint32_t ql[17], qh[9], sc[3]; uint32_t d, sh; };
            auto load = [&](int hb, Raw& w) {
                const uint8_t* blk = row + (size_t)(hb >> 1) * GB_Q6K_BYTES;
                const int h = hb & 1;
                const uint32_t* pl = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk + 64 * h) & ~uintptr_t(3));
                const uint32_t* ph = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk + 128 + 32 * h) & ~uintptr_t(3));
                const uint32_t* ps = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk + 192 + 8 * h) & ~uintptr_t(3));
#pragma unroll
                for (int i = 0; i < 17; i++) w.ql[i] = __ldg(pl + i);   // within the block: ends by byte 132
#pragma unroll
                for (int i = 0; i < 9; i++) w.qh[i] = __ldg(ph + i);    // ends by byte 196
                w.sc[0] = __ldg(ps);
                w.sc[1] = __ldg(ps + 1);
                // a third word only when the scales start 2 bytes into a word (it then ends at byte 210)
                w.sc[2] = (reinterpret_cast<uintptr_t>(blk) & 3) ? __ldg(ps + 2) : 0u;
                w.d = *reinterpret_cast<const uint16_t*>(blk + 208);
                w.sh = (uint32_t)((reinterpret_cast<uintptr_t>(blk) & 3) * 8);   // 0 or 16 (blocks are 2-byte aligned)
            };
            Raw cur, nxt;
            load(0, cur);
            for (int hb = 0; hb < nk / 4; hb++) {
                if (hb + 1 < nk / 4) load(hb + 1, nxt);
                uint32_t ql[16], qh[8], scw[2];
                const uint32_t sh = cur.sh;
#pragma unroll
                for (int i = 0; i < 16; i++) ql[i] = __funnelshift_r(cur.ql[i], cur.ql[i + 1], sh);
#pragma unroll
                for (int i = 0; i < 8; i++) qh[i] = __funnelshift_r(cur.qh[i], cur.qh[i + 1], sh);
                scw[0] = __funnelshift_r(cur.sc[0], cur.sc[1], sh);
                scw[1] = __funnelshift_r(cur.sc[1], cur.sc[2], sh);
                const float d = f16_bits_to_f32(cur.d);
#pragma unroll
                for (int G = 0; G < 4; G++) {
                    const int s0 = (int)(int8_t)((scw[G >> 1] >> (16 * (G & 1))) & 0xFF);
                    const int s1 = (int)(int8_t)((scw[G >> 1] >> (16 * (G & 1) + 8)) & 0xFF);
                    const float ds0 = d * (float)s0 * rs, ds1 = d * (float)s1 * rs;
                    float v[32];
#pragma unroll
                    for (int wi = 0; wi < 8; wi++) {
                        const uint32_t lo4 = (ql[8 * (G & 1) + wi] >> (4 * (G >> 1))) & 0x0F0F0F0Fu;
                        const uint32_t hi2 = ((qh[wi] >> (2 * G)) & 0x03030303u) << 4;
                        const uint32_t qw = lo4 | hi2;   // 4 six-bit codes, one per byte
                        const float dsw = wi < 4 ? ds0 : ds1;
                        v[4 * wi + 0] = dsw * tc::byte_as_float<0>(qw, 32.f);
                        v[4 * wi + 1] = dsw * tc::byte_as_float<1>(qw, 32.f);
                        v[4 * wi + 2] = dsw * tc::byte_as_float<2>(qw, 32.f);
                        v[4 * wi + 3] = dsw * tc::byte_as_float<3>(qw, 32.f);
                    }
                    if (n >= N) {
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = 0.f;
                    }
                    put(4 * hb + G, v);
                }
                cur = nxt;
            }
        } else {
            for (int kc = 0; kc < nk; kc++) {
                float v[32];
                if (n < N) {
                    dequant32<DT>(Wm, n, K, kc * GM_BK, v);
                    if constexpr (H16) {
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] *= rs;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = 0.f;
                }
                put(kc, v);
            }
        }
    } else if (warp == GM_XPROD) {   // ---- activation tiles by TMA
        if (lane == 0) {
            bool ok = true;
            for (int kc = 0; kc < nk && ok; kc++) {
                const int s = kc % C::S;
                if (kc >= C::S) ok = gm_wait(empty + 8 * s, ((kc / C::S) - 1) & 1, err);
                if (!ok) break;
                if constexpr (H16) {
                    // the hi and lo tiles [BT tokens][32] in the K-major
                    // layout, completing on the stage's "full" barrier
                    const uint32_t b = tc::smem_u32(smem + (size_t)s * C::STAGE + 2 * C::TILE_A);
                    mbs_expect(full + 8 * s, 2 * C::TILE_B);
                    tma_load_3d(b, &xmap, 0, t0 / 128, kc * (GM_BK / 8), full + 8 * s);
                    tma_load_3d(b + C::TILE_B, &xlmap, 0, t0 / 128, kc * (GM_BK / 8), full + 8 * s);
                    continue;
                }
                // raw fp32 [BT tokens][32]
                mbs_expect(xfull + 8 * s, C::XRAW);
                // into the stage's B tiles; rows past T read as zeros
                tma_load_3d(tc::smem_u32(smem + (size_t)s * C::STAGE + 2 * C::TILE_A), &xmap, kc * GM_BK, t0, 0,
                            xfull + 8 * s);
            }
        }
        __syncwarp();
    } else if (warp >= 5 + GM_READERS) {   // ---- tf32: split the raw activation tile in place
      if constexpr (!H16) {
        // lane (qq, j) converts row xw * 32 + 8 qq + j; step c takes its
        // column group (j + c) mod 8, so a quarter-warp's 16-byte reads (one
        // raw row each) and writes (one core matrix) hit 8 different bank groups
        const int xw = warp - (5 + GM_READERS), j = lane & 7;
        const int rr = xw * 32 + 8 * (lane >> 3) + j;
        constexpr int NP = BT / 128;   // 128-row passes (the warp's rows rr + 128 pass)
        bool ok = true;
        for (int kc = 0; kc < nk; kc++) {
            const int s = kc % C::S;
            if (ok) ok = gm_wait(xfull + 8 * s, (kc / C::S) & 1, err);
            uint8_t* hi = smem + (size_t)s * C::STAGE + 2 * C::TILE_A;
            float4 u[NP][8];
#pragma unroll
            for (int pp = 0; pp < NP; pp++)
#pragma unroll
                for (int c = 0; c < 8; c++)
                    u[pp][c] = *reinterpret_cast<const float4*>(hi + (rr + 128 * pp) * 128 + ((j + c) & 7) * 16);
            // every raw row is read before any core matrix overwrites it
            asm volatile("bar.sync 1, %0;" ::"n"(GM_XWARPS * 32) : "memory");
#pragma unroll
            for (int pp = 0; pp < NP; pp++)
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    float h[4], l[4];
                    tc::split_tf32(u[pp][c].x, h[0], l[0]);
                    tc::split_tf32(u[pp][c].y, h[1], l[1]);
                    tc::split_tf32(u[pp][c].z, h[2], l[2]);
                    tc::split_tf32(u[pp][c].w, h[3], l[3]);
                    const uint32_t off = tc::tile_off(rr + 128 * pp, 4 * ((j + c) & 7), BT);
                    *reinterpret_cast<float4*>(hi + off) = make_float4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<float4*>(hi + C::TILE_B + off) = make_float4(l[0], l[1], l[2], l[3]);
                }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) mbs_arrive(full + 8 * s);
        }
      }
    } else {   // ---- warps 5-8: sum the accumulators in fp32, then write Y
        // lane r of warp w reads tensor-memory lane 32 (w % 4) + r = weight
        // row; the running sum lives in a third tensor-memory region
        const int q = warp & 3;
        const int r = q * 32 + lane, n = SW ? n0 + (r & 63) : n0 + r;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        constexpr int XLD = BT + 1;   // SW: final sums [128 rows][BT] in the (then idle) stage memory
        float* xch = reinterpret_cast<float*>(smem);
        const uint32_t sum = lane_base + (uint32_t)(C::NACC * BT);
        // fp16 operands: 2^-e_n of this weight row (times 2^-e_t per token below)
        const float inv_r = H16 && n < N ? tc::pow2f(-row_scale_exp<DT>((SW && r >= 64) ? W2 : W, n, K)) : 1.f;
        bool ok = true;
        for (int g = 0; g < ng && ok; g++) {
            const int a = g % C::NACC;
            ok = gm_wait(accfull + 8 * a, (g / C::NACC) & 1, err);
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t acc = lane_base + (uint32_t)(a * BT);
            const bool last = g == ng - 1;
#pragma unroll 1
            for (int c = 0; c < BT; c += 32) {
                float v[32];
                if (g > 0) {
                    float u[32];
                    tc::tmem_ld32x2(acc + c, sum + c, v, u);
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] += u[i];
                } else {
                    tc::tmem_ld32(acc + c, v);
                }
                if (!last) {
                    tc::tmem_st32_nowait(sum + c, v);
                    continue;
                }
                if constexpr (H16) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int tt = t0 + c + i;
                        v[i] = v[i] * inv_r * (tt < T ? xinv[tt] : 1.f);
                    }
                }
                if constexpr (SW) {
#pragma unroll
                    for (int i = 0; i < 32; i++) xch[r * XLD + c + i] = v[i];
                } else if (n < N) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int tt = t0 + c + i;
                        if (tt < T) {
                            const size_t o = (size_t)tt * ldy + n;
                            Y[o] = v[i] + (R ? R[o] : 0.f);
                        }
                    }
                }
            }
            if (!last) tc::tmem_wait_st();   // the running sum is read back by the next group
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbs_arrive(accfree + 8 * a);
        }
        if constexpr (SW) {
            // every MMA has completed (the last group's commit), so the stages
            // are idle; gate row i pairs with up row 64 + i
            asm volatile("bar.sync 2, %0;" ::"n"(GM_READERS * 32) : "memory");
            const int rt = (warp - 5) * 32 + lane;
            for (int idx = rt; idx < 64 * BT && ok; idx += GM_READERS * 32) {
                const int fi = idx & 63, tl = idx >> 6, f = n0 + fi, tt = t0 + tl;
                if (f < N && tt < T) {
                    const float x = xch[fi * XLD + tl], u = xch[(64 + fi) * XLD + tl];
                    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));   // k_silu_mul (kernels_cpu.c:323-336)
                    Y[(size_t)tt * ldy + f] = __fmul_rn(__fmul_rn(x, sig), u);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 4) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Split 8 token rows of X per CTA (K a multiple of 32) for fp16 operands:
// e from each row's largest |x| (so that |x| 2^e < 2^15; one warp per row),
// then x 2^e = hi + lo as fp16 halves (tc::split_f16x2) written
// column-group-major (8 rows x 16 bytes: one 128-byte line per group), inv =
// 2^-e; rows T .. tp - 1 are zero.  Non-negative floats order as their bit
// patterns.
constexpr int XS_ROWS = 8;
__global__ void __launch_bounds__(256) k_x_split16(const float* __restrict__ X, int K, int T, int tp,
                                                    uint4* __restrict__ hi, uint4* __restrict__ lo,
                                                    float* __restrict__ inv) {
    __shared__ float scale[XS_ROWS];
    const int t0 = blockIdx.x * XS_ROWS, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int rr = warp; rr < XS_ROWS; rr += 8) {   // a row per warp
        const int t = t0 + rr;
        uint32_t m = 0;
        if (t < T) {
            const float4* row = reinterpret_cast<const float4*>(X + (size_t)t * K);
            for (int i = lane; i < K / 4; i += 32) {
                const float4 v = __ldg(row + i);
                m = max(m, max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                               max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w)))));
            }
        }
        m = __reduce_max_sync(0xFFFFFFFFu, m);
        if (lane == 0) {
            const int e = tc::f16_scale_exp(m);
            scale[rr] = tc::pow2f(e);
            if (t < T) inv[t] = tc::pow2f(-e);
        }
    }
    __syncthreads();
    const int ng = K / 8;
    for (int idx = threadIdx.x; idx < ng * XS_ROWS; idx += blockDim.x) {
        const int rr = idx % XS_ROWS, g = idx / XS_ROWS, t = t0 + rr;
        uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
        if (t < T) {
            const float4* p = reinterpret_cast<const float4*>(X + (size_t)t * K + 8 * g);
            const float4 a = __ldg(p), b = __ldg(p + 1);
            const float sc = scale[rr];
            tc::split_f16x2(a.x * sc, a.y * sc, h.x, l.x);
            tc::split_f16x2(a.z * sc, a.w * sc, h.y, l.y);
            tc::split_f16x2(b.x * sc, b.y * sc, h.z, l.z);
            tc::split_f16x2(b.z * sc, b.w * sc, h.w, l.w);
        }
        const size_t o = (size_t)g * tp + t;
        hi[o] = h;
        lo[o] = l;
    }
}

// RMSNorm of 8 token rows per CTA fused with their split: xn = w * (x * r),
// r = 1 / sqrt(sum(x^2) / K + eps) (kernels_cpu.c:242-263, k_rmsnorm's
// roundings; the sum of squares in another order), then split as
// k_x_split16 does.  xn itself is not written.
__global__ void __launch_bounds__(256) k_rmsnorm_split16(const float* __restrict__ X, const float* __restrict__ w,
                                                          int K, float eps, int T, int tp, uint4* __restrict__ hi,
                                                          uint4* __restrict__ lo, float* __restrict__ inv) {
    __shared__ float scale[XS_ROWS], rsq[XS_ROWS];
    const int t0 = blockIdx.x * XS_ROWS, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int rr = warp; rr < XS_ROWS; rr += 8) {   // a row per warp
        const int t = t0 + rr;
        float r = 0.f;
        uint32_t m = 0;
        if (t < T) {
            const float4* row = reinterpret_cast<const float4*>(X + (size_t)t * K);
            float ss = 0.f;
            for (int i = lane; i < K / 4; i += 32) {
                const float4 v = __ldg(row + i);
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
            r = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
            for (int i = lane; i < K / 4; i += 32) {
                const float4 v = __ldg(row + i);
                const float4 g = w ? __ldg(w4 + i) : make_float4(1.f, 1.f, 1.f, 1.f);
                m = max(m, max(max(__float_as_uint(fabsf(__fmul_rn(g.x, __fmul_rn(v.x, r)))),
                                   __float_as_uint(fabsf(__fmul_rn(g.y, __fmul_rn(v.y, r))))),
                               max(__float_as_uint(fabsf(__fmul_rn(g.z, __fmul_rn(v.z, r)))),
                                   __float_as_uint(fabsf(__fmul_rn(g.w, __fmul_rn(v.w, r)))))));
            }
        }
        m = __reduce_max_sync(0xFFFFFFFFu, m);
        if (lane == 0) {
            const int e = tc::f16_scale_exp(m);
            scale[rr] = tc::pow2f(e);
            rsq[rr] = r;
            if (t < T) inv[t] = tc::pow2f(-e);
        }
    }
    __syncthreads();
    const int ng = K / 8;
    for (int idx = threadIdx.x; idx < ng * XS_ROWS; idx += blockDim.x) {
        const int rr = idx % XS_ROWS, g = idx / XS_ROWS, t = t0 + rr;
        uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
        if (t < T) {
            const float4* p = reinterpret_cast<const float4*>(X + (size_t)t * K + 8 * g);
            const float4 a = __ldg(p), b = __ldg(p + 1);
            const float4 ga = w ? __ldg(w4 + 2 * g) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 gb = w ? __ldg(w4 + 2 * g + 1) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float r = rsq[rr], sc = scale[rr];
            auto nv = [&](float x, float gg) { return __fmul_rn(gg, __fmul_rn(x, r)) * sc; };
            tc::split_f16x2(nv(a.x, ga.x), nv(a.y, ga.y), h.x, l.x);
            tc::split_f16x2(nv(a.z, ga.z), nv(a.w, ga.w), h.y, l.y);
            tc::split_f16x2(nv(b.x, gb.x), nv(b.y, gb.y), h.z, l.z);
            tc::split_f16x2(nv(b.z, gb.z), nv(b.w, gb.w), h.w, l.w);
        }
        const size_t o = (size_t)g * tp + t;
        hi[o] = h;
        lo[o] = l;
    }
}

int gemm_rmsnorm_split_x(const float* X, const float* w, int T, int K, float eps, void* hi, void* lo, float* inv,
                         cudaStream_t st) {
    if (!X || !hi || !lo || !inv || T <= 0 || K <= 0 || K % 32 || (reinterpret_cast<uintptr_t>(X) & 15) ||
        (w && (reinterpret_cast<uintptr_t>(w) & 15)) || (reinterpret_cast<uintptr_t>(hi) & 15) ||
        (reinterpret_cast<uintptr_t>(lo) & 15))
        return GB_EINVAL;
    const int tp = gemm_split_rows(T);
    k_rmsnorm_split16<<<tp / XS_ROWS, 256, 0, st>>>(X, w, K, eps, T, tp, static_cast<uint4*>(hi),
                                                    static_cast<uint4*>(lo), inv);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

bool gemm_f16_operands() {
    static const bool f16 = [] {
        const char* e = getenv("GB_GEMM_KIND");
        return !(e && strcmp(e, "tf32") == 0);
    }();
    return f16;
}

int gemm_split_x(const float* X, int T, int K, void* hi, void* lo, float* inv, cudaStream_t st) {
    if (!X || !hi || !lo || !inv || T <= 0 || K <= 0 || K % 32 || (reinterpret_cast<uintptr_t>(X) & 15) ||
        (reinterpret_cast<uintptr_t>(hi) & 15) || (reinterpret_cast<uintptr_t>(lo) & 15))
        return GB_EINVAL;
    const int tp = gemm_split_rows(T);
    k_x_split16<<<tp / XS_ROWS, 256, 0, st>>>(X, K, T, tp, static_cast<uint4*>(hi), static_cast<uint4*>(lo), inv);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

template <int DT, int BT, bool SW, bool H16>
static int launch_gemm_bt(const void* W, const void* W2, const float* X, float* Y, const float* R, const GemmX16* x16,
                          int N, int ldy, int K, int T, cudaStream_t st, unsigned* err) {
    using C = GmCfg<BT, H16>;
    static_assert(!SW || 128 * (BT + 1) * 4 <= C::S * C::STAGE, "SwiGLU exchange fits the stages");
    GB_CUDA_TRY(set_smem_once(reinterpret_cast<const void*>(k_gemm<DT, BT, SW, H16>), C::SMEM));
    CUtensorMap xmap, xlmap;
    const float* xinv = nullptr;
    if constexpr (H16) {
        if (x16->tp < gemm_split_rows(T) || !gemm_encode_x16(&xmap, x16->hi, x16->tp, K, BT) ||
            !gemm_encode_x16(&xlmap, x16->lo, x16->tp, K, BT))
            return GB_ECUDA;
        xinv = x16->inv;
    } else {
        if (!gemm_encode_x(&xmap, X, T, K, GM_BK, BT)) return GB_ECUDA;
        xlmap = xmap;
    }
    const int rows = SW ? GM_ROWS / 2 : GM_ROWS;
    dim3 grid((N + rows - 1) / rows, (T + BT - 1) / BT);
    k_gemm<DT, BT, SW, H16><<<grid, GM_THREADS, C::SMEM, st>>>(
        xmap, static_cast<const uint8_t*>(W), static_cast<const uint8_t*>(W2), Y, R, xlmap, xinv, N, ldy, K, T, err);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

// 256-token tiles (half the MMA instructions and weight conversions per
// FLOP) when their grid still gives every SM a CTA, else 128-token tiles
// (GB_GEMM_BT=128 / 256 forces one size).
template <int DT, bool SW>
static int launch_gemm(const void* W, const void* W2, const float* X, float* Y, const float* R, const GemmX16* x16,
                       int N, int ldy, int K, int T, cudaStream_t st, unsigned* err) {
    static const int force = [] {
        const char* e = getenv("GB_GEMM_BT");
        return e ? atoi(e) : 0;
    }();
    const int rows = SW ? GM_ROWS / 2 : GM_ROWS;
    const long ctas256 = (long)((N + rows - 1) / rows) * ((T + 255) / 256);
    const bool wide = force ? force == 256 : ctas256 >= sm_count();
    if (x16)
        return wide ? launch_gemm_bt<DT, 256, SW, true>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err)
                    : launch_gemm_bt<DT, 128, SW, true>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err);
    return wide ? launch_gemm_bt<DT, 256, SW, false>(W, W2, X, Y, R, nullptr, N, ldy, K, T, st, err)
                : launch_gemm_bt<DT, 128, SW, false>(W, W2, X, Y, R, nullptr, N, ldy, K, T, st, err);
}

template <bool SW>
static int gemm_dispatch(int dtype, const void* W, const void* W2, const float* X, float* Y, const float* R, int N,
                         int ldy, int K, int T, cudaStream_t st, unsigned* err, const GemmX16* x16) {
    if (!W || (!X && !x16) || !Y || N <= 0 || K <= 0 || T <= 0 || ldy < N || (SW && !W2)) return GB_EINVAL;
    if (x16 && (!x16->hi || !x16->lo || !x16->inv)) return GB_EINVAL;
    const bool a16 = dtype == GB_DT_F32 || dtype == GB_DT_Q4_K || dtype == GB_DT_Q5_K || dtype == GB_DT_F16;
    if ((reinterpret_cast<uintptr_t>(X) & 15) ||
        (a16 && ((reinterpret_cast<uintptr_t>(W) & 15) || (SW && (reinterpret_cast<uintptr_t>(W2) & 15)))))
        return GB_EINVAL;
    if (dtype != GB_DT_F32 && dtype != GB_DT_Q8_0 && dtype != GB_DT_Q4_K && dtype != GB_DT_Q6_K &&
        dtype != GB_DT_Q5_K && dtype != GB_DT_F16)
        return GB_EINVAL;
    const int kmul = (dtype == GB_DT_Q4_K || dtype == GB_DT_Q6_K || dtype == GB_DT_Q5_K) ? 256 : 32;
    if (K % kmul) return GB_ESHAPE;
    if (!gemm_f16_operands()) {
        if (!X) return GB_EINVAL;   // a split X needs the fp16 form
        x16 = nullptr;
    }
    // fp16 operands without the caller's split: X split here into
    // stream-ordered scratch (hi, lo, inv)
    void* tmp = nullptr;
    GemmX16 own;
    if (gemm_f16_operands() && !x16) {
        const size_t half = (size_t)gemm_split_rows(T) * K * 2;
        if (cudaMallocAsync(&tmp, 2 * half + (size_t)T * sizeof(float), st) != cudaSuccess) return GB_ENOMEM;
        uint8_t* b = static_cast<uint8_t*>(tmp);
        own.hi = b;
        own.lo = b + half;
        own.inv = reinterpret_cast<const float*>(b + 2 * half);
        own.tp = gemm_split_rows(T);
        const int rc = gemm_split_x(X, T, K, b, b + half, reinterpret_cast<float*>(b + 2 * half), st);
        if (rc) {
            cudaFreeAsync(tmp, st);
            return rc;
        }
        x16 = &own;
    }
    int rc;
    switch (dtype) {
        case GB_DT_F32: rc = launch_gemm<GB_DT_F32, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
        case GB_DT_Q8_0: rc = launch_gemm<GB_DT_Q8_0, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
        case GB_DT_Q4_K: rc = launch_gemm<GB_DT_Q4_K, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
        case GB_DT_Q6_K: rc = launch_gemm<GB_DT_Q6_K, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
        case GB_DT_Q5_K: rc = launch_gemm<GB_DT_Q5_K, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
        default: rc = launch_gemm<GB_DT_F16, SW>(W, W2, X, Y, R, x16, N, ldy, K, T, st, err); break;
    }
    if (tmp && cudaFreeAsync(tmp, st) != cudaSuccess && rc == GB_OK) rc = GB_ECUDA;
    return rc;
}

int gemm_launch(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T,
                cudaStream_t st, unsigned* err, int ldy, const GemmX16* x16) {
    return gemm_dispatch<false>(dtype, W, nullptr, X, Y, R, N, ldy ? ldy : N, K, T, st, err, x16);
}

int gemm_swiglu_launch(int dtype, const void* Wg, const void* Wu, const float* X, float* Y, int F, int K, int T,
                       cudaStream_t st, unsigned* err, int ldy, const GemmX16* x16) {
    return gemm_dispatch<true>(dtype, Wg, Wu, X, Y, nullptr, F, ldy ? ldy : F, K, T, st, err, x16);
}

}  // namespace gb

extern "C" int gb_gemm(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T,
                       void* stream) {
    return gb::gemm_launch(dtype, W, X, Y, R, N, K, T, static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" size_t gb_gemm_split_bytes(int T, int K) {
    return T > 0 && K > 0 ? (size_t)gb::gemm_split_rows(T) * K * 2 : 0;
}

extern "C" int gb_gemm_split(const float* X, int T, int K, void* hi, void* lo, float* inv, void* stream) {
    if (!gb::gemm_f16_operands()) return GB_EINVAL;
    return gb::gemm_split_x(X, T, K, hi, lo, inv, static_cast<cudaStream_t>(stream));
}

extern "C" int gb_gemm_presplit(int dtype, const void* W, const void* hi, const void* lo, const float* inv, float* Y,
                                const float* R, int N, int K, int T, void* stream) {
    if (!gb::gemm_f16_operands() || T <= 0) return GB_EINVAL;
    const gb::GemmX16 x16{hi, lo, inv, gb::gemm_split_rows(T)};
    return gb::gemm_launch(dtype, W, nullptr, Y, R, N, K, T, static_cast<cudaStream_t>(stream), nullptr, 0, &x16);
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
