// gb_prefill.cu -- a prompt of T tokens through one transformer layer at
// once: the T > 1 branch of the reference's transformer_layer
// (src/engine/engine.c:353-546), which the reference runs on its CPU kernels
// (its GPU prefill hook, src/engine/gpu_prefill.c:3-20, is a stub).
//
//   xn = RMSNorm(h) rows            k_rmsnorm, one CTA per row
//   q, k, v = xn . W^T              gb_gemm (tcgen05, 3xTF32)
//   RoPE(q), RoPE(k), KV append     k_pf_rope_kv (rows pos0 .. pos0 + T - 1)
//   attn = causal softmax(q k^T / sqrt(hd)) v    k_pf_attn
//   h += attn . Wo^T                gb_gemm with the residual
//   xn = RMSNorm(h)                 k_rmsnorm
//   gate = silu(xn Wg^T) * (xn Wu^T)  one GEMM launch (gate and up rows per CTA)
//   h += gate . Wdown^T             gb_gemm with the residual
//
// Activations are row-major [T][width] fp32 in HBM; the K / V caches keep the
// decode layout [n_kv][max_seq][hd], so decode continues from pos0 + T.
#include "gb_common.cuh"
#include "gb_internal.h"
#include "gb_mt.cuh"
#include "gb_tc.cuh"

#include <stdlib.h>
#include <string.h>

namespace gb {

__device__ unsigned g_pf_err;   // bounded-wait timeouts of gb_prefill_attention (no model error word)

// ---------------------------------------------------------------- RoPE + KV append
// Row t (position pos0 + t): q heads rotated in place, k heads rotated into
// the K cache, v copied into the V cache.  Same rotation and rounding as the
// decode attention (kernels_cpu.c:391-431: a c - b s, a s + b c).
__global__ void __launch_bounds__(256) k_pf_rope_kv(float* __restrict__ q, const float* __restrict__ k,
                                                    const float* __restrict__ v, float* __restrict__ kc,
                                                    float* __restrict__ vc, const float* __restrict__ rope, int pos0,
                                                    int nh, int nkv, int hd, int max_seq) {
    const int t = blockIdx.x, pos = pos0 + t, half = hd / 2;
    const int QD = nh * hd, KVD = nkv * hd;
    const float* cs = rope + (size_t)pos * hd;
    for (int e = threadIdx.x; e < (nh + nkv) * half; e += blockDim.x) {
        const int h = e / half, i = e % half;
        const float* src;
        float* dst;
        if (h < nh) {
            src = dst = q + (size_t)t * QD + (size_t)h * hd;
        } else {
            src = k + (size_t)t * KVD + (size_t)(h - nh) * hd;
            dst = kc + ((size_t)(h - nh) * max_seq + pos) * hd;
        }
        const float a = src[2 * i], b = src[2 * i + 1], c = cs[2 * i], s = cs[2 * i + 1];
        dst[2 * i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        dst[2 * i + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    for (int e = threadIdx.x; e < KVD; e += blockDim.x)
        vc[((size_t)(e / hd) * max_seq + pos) * hd + e % hd] = v[(size_t)t * KVD + e];
}

// ---------------------------------------------------------------- causal attention
// One CTA: KV head g and a block of BQ query rows for each of its GROUP query
// heads (PA_R = 64 (head, query) rows in all), so every K / V tile read from
// the cache serves all the heads that share it.  Keys stream in tiles of 64
// through a two-stage cp.async ring; scores, the online softmax (running max
// and sum per row, as flash attention does) and P.V run on the fp32 CUDA
// cores (packed two-wide FMAs).  Thread (tr, tc) owns rows tr + 16 i and keys
// tc + 16 j of a tile (i, j < 4) and output columns 4 tc + 64 c .. + 3.  The reference's order
// (engine.c:431-500: scores * scale, -inf above the diagonal, softmax,
// scores . V) is kept; only the summation order differs.
constexpr int PA_R = 64;        // (head, query) rows per CTA
constexpr int PA_BK = 64;       // keys per tile
constexpr int PA_THREADS = 256;

template <int HD>
constexpr int pa_smem_bytes() {
    return (PA_R * (HD + 4) + 2 * 2 * PA_BK * (HD + 4) + PA_BK * (PA_R + 4)) * 4;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <int HD, int GROUP>
__global__ void __launch_bounds__(PA_THREADS) k_pf_attn(const float* __restrict__ q, const float* __restrict__ kc,
                                                        const float* __restrict__ vc, float* __restrict__ out, int T,
                                                        int pos0, int nh, int max_seq) {
    constexpr int LD = HD + 4, BQ = PA_R / GROUP, LP = PA_R + 4, NC = HD / 64;
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                          // [PA_R][LD]
    float* Ks = Qs + PA_R * LD;              // [2][PA_BK][LD]
    float* Vs = Ks + 2 * PA_BK * LD;         // [2][PA_BK][LD]
    float* Ps = Vs + 2 * PA_BK * LD;         // [PA_BK][LP], rows permuted: row tr + 16 i at tr * 4 + i
    const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
    const int g = blockIdx.y;
    const int nqb = gridDim.x, qb = nqb - 1 - blockIdx.x;   // longest blocks first
    const int q0 = qb * BQ;
    const int QD = nh * HD;
    const float* kh = kc + (size_t)g * max_seq * HD;
    const float* vh = vc + (size_t)g * max_seq * HD;
    const int kend = pos0 + min(q0 + BQ, T);   // keys 0 .. kend - 1 (the last query row's causal range)
    const int nt = (kend + PA_BK - 1) / PA_BK;

    // Q rows: row r = head g * GROUP + r / BQ, query q0 + r % BQ (zero past T)
    for (int e = tid; e < PA_R * HD / 4; e += PA_THREADS) {
        const int r = e / (HD / 4), d4 = e % (HD / 4);
        const int t = q0 + r % BQ, h = g * GROUP + r / BQ;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < T) val = *reinterpret_cast<const float4*>(q + (size_t)t * QD + (size_t)h * HD + 4 * d4);
        *reinterpret_cast<float4*>(Qs + r * LD + 4 * d4) = val;
    }
    auto load_tile = [&](int kt, int b) {
        const uint32_t kb = (uint32_t)__cvta_generic_to_shared(Ks + b * PA_BK * LD);
        const uint32_t vb = (uint32_t)__cvta_generic_to_shared(Vs + b * PA_BK * LD);
        for (int e = tid; e < PA_BK * HD / 4; e += PA_THREADS) {
            const int r = e / (HD / 4), d4 = e % (HD / 4), key = kt * PA_BK + r;
            const bool in = key < kend;   // rows past the causal range are zero-filled
            const size_t off = (size_t)(in ? key : 0) * HD + 4 * d4;
            const uint32_t so = (uint32_t)((r * LD + 4 * d4) * 4);
            cp_async16(kb + so, kh + off, in ? 16 : 0);
            cp_async16(vb + so, vh + off, in ? 16 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_tile(0, 0);

    const float scale = 1.0f / sqrtf((float)HD);
    int qpos[4];
#pragma unroll
    for (int i = 0; i < 4; i++) qpos[i] = pos0 + q0 + (tr + 16 * i) % BQ;
    float m[4], l[4], o[4][4 * NC];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 4 * NC; c++) o[i][c] = 0.f;
    }
    for (int kt = 0; kt < nt; kt++) {
        const int b = kt & 1;
        if (kt + 1 < nt) {
            load_tile(kt + 1, b ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float* Kb = Ks + b * PA_BK * LD;
        const float* Vb = Vs + b * PA_BK * LD;
        // ---- scores
        // two partial sums per score (even / odd columns), two FMAs per
        // packed instruction
        float2 s2[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s2[i][j] = make_float2(0.f, 0.f);
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4*>(Qs + (tr + 16 * i) * LD + d);
#pragma unroll
            for (int j = 0; j < 4; j++) kv[j] = *reinterpret_cast<const float4*>(Kb + (tc + 16 * j) * LD + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    s2[i][j] = __ffma2_rn(make_float2(qv[i].x, qv[i].y), make_float2(kv[j].x, kv[j].y), s2[i][j]);
                    s2[i][j] = __ffma2_rn(make_float2(qv[i].z, qv[i].w), make_float2(kv[j].z, kv[j].w), s2[i][j]);
                }
        }
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = s2[i][j].x + s2[i][j].y;
        // ---- scale, causal mask, online softmax
        float p[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int key = kt * PA_BK + tc + 16 * j;
                s[i][j] = key > qpos[i] ? -INFINITY : s[i][j] * scale;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);   // finite: key 0 is in every row's range
            const float alpha = expf(m[i] - mn);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                p[i][j] = expf(s[i][j] - mn);
                sum += p[i][j];
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = fmaf(l[i], alpha, sum);
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < 4 * NC; c++) o[i][c] *= alpha;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4*>(Ps + (tc + 16 * j) * LP + tr * 4) = make_float4(p[0][j], p[1][j], p[2][j], p[3][j]);
        __syncthreads();
        // ---- o += P . V
#pragma unroll 4
        for (int kk = 0; kk < PA_BK; kk++) {
            const float4 pv = *reinterpret_cast<const float4*>(Ps + kk * LP + tr * 4);
            const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int c = 0; c < NC; c++) {
                const float4 vv = *reinterpret_cast<const float4*>(Vb + kk * LD + 64 * c + 4 * tc);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 pp = make_float2(pr[i], pr[i]);
                    float2 lo = __ffma2_rn(pp, make_float2(vv.x, vv.y), make_float2(o[i][4 * c], o[i][4 * c + 1]));
                    float2 hi = __ffma2_rn(pp, make_float2(vv.z, vv.w), make_float2(o[i][4 * c + 2], o[i][4 * c + 3]));
                    o[i][4 * c] = lo.x;
                    o[i][4 * c + 1] = lo.y;
                    o[i][4 * c + 2] = hi.x;
                    o[i][4 * c + 3] = hi.y;
                }
            }
        }
        __syncthreads();   // the tile buffer and P are rewritten next
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = tr + 16 * i, t = q0 + r % BQ, h = g * GROUP + r / BQ;
        if (t >= T) continue;
        const float inv = 1.0f / l[i];
        float* dst = out + (size_t)t * QD + (size_t)h * HD;
#pragma unroll
        for (int c = 0; c < NC; c++)
            *reinterpret_cast<float4*>(dst + 64 * c + 4 * tc) =
                make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv, o[i][4 * c + 2] * inv, o[i][4 * c + 3] * inv);
    }
}

template <int HD, int GROUP>
static cudaError_t launch_pf_attn(const float* q, const float* kc, const float* vc, float* out, int T, int pos0,
                                  int n_kv, int max_seq, cudaStream_t st) {
    constexpr int smem = pa_smem_bytes<HD>();
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(k_pf_attn<HD, GROUP>), smem);
    if (e != cudaSuccess) return e;
    constexpr int BQ = PA_R / GROUP;
    dim3 grid((T + BQ - 1) / BQ, n_kv);
    k_pf_attn<HD, GROUP><<<grid, PA_THREADS, smem, st>>>(q, kc, vc, out, T, pos0, n_kv * GROUP, max_seq);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- causal attention on the tensor cores
// One CTA: KV head g and TA_R = 128 (head, query) rows (GROUP heads x 128 /
// GROUP queries), keys in tiles of TA_NK = 64.  3xTF32 as the GEMM (gb_gemm.cu):
// every operand is split into a tf32 part and an fp32 remainder and the
// tensor cores sum hi.hi + hi.lo + lo.hi.
//   S = Q K^T   A = Q, resident in tensor memory as hi / lo (lane = row,
//               head_dim columns each), B = the K tile in shared memory
//               (N 64 keys x K head_dim); S in tensor memory, double-buffered
//               so S(t + 1) is computed during softmax(t)
//   softmax     warps 0-3, thread = row = tensor-memory lane: the scores
//               scaled and masked as the reference does (engine.c:431-500),
//               running max and sum (online softmax, the max moved only when
//               exceeded by more than TA_TAU); P = exp(s - m) split into
//               shared memory; O (tensor memory) rescaled by exp(m_old -
//               m_new) before the next P.V accumulates into it, when m moved
//   O += P V    A = P (M 128 x K 64), B = V^T (N hd x K 64: the converters
//               transpose the V tile)
// Tensor memory: Q hi [0, hd), Q lo [hd, 2 hd), S[2] at 2 hd + 0 / 64, O at
// 2 hd + 128 (512 columns at hd 128).  Warps 4-7 convert the K / V tiles
// (read from the cache, L2-resident); warp 8 owns the tensor memory and one
// lane issues the MMAs.  Every wait is bounded and records GB_ETIMEOUT.
constexpr int TA_R = 128;
constexpr int TA_NK = 64;
constexpr int TA_THREADS = 9 * 32;
constexpr float TA_TAU = 8.0f;   // a row's max moves (O, l rescaled) only when exceeded by this much

template <int HD>
struct TaLayout {
    static constexpr int NS = HD / 32;                    // 32-column sub-tiles along head_dim
    static constexpr int KSUB = TA_NK * 32 * 4;           // K: [64 keys x 32] sub-tile (8 KB)
    static constexpr int VSUB = HD * 32 * 4;              // V^T: [hd x 32 keys] sub-tile
    static constexpr int PSUB = TA_R * 32 * 4;            // P: [128 x 32 keys] sub-tile (16 KB)
    static constexpr int K_HI = 0, K_LO = NS * KSUB;
    static constexpr int V_HI = 2 * NS * KSUB, V_LO = V_HI + 2 * VSUB;
    static constexpr int P_HI = V_LO + 2 * VSUB, P_LO = P_HI + 2 * PSUB;
    static constexpr int BYTES = P_LO + 2 * PSUB;
    static constexpr int SMEM = BYTES + 1024;             // + alignment slack
    static constexpr uint32_t QHI = 0, QLO = HD, S0 = 2 * HD, OC = 2 * HD + 128;   // tensor-memory columns
    static constexpr uint32_t TMEM_COLS = 512;
};
static_assert(TaLayout<128>::SMEM <= 227 * 1024, "shared memory");
static_assert(TaLayout<128>::OC + 128 <= TaLayout<128>::TMEM_COLS, "tensor memory");

__device__ __forceinline__ bool ta_wait(uint32_t bar, uint32_t parity, unsigned* err) {
    if (mbs_test(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbs_test(bar, parity))
        if (gtimer() - t0 > MT_WAIT_NS) {
            atomicExch(err, (unsigned)(-GB_ETIMEOUT));
            return false;
        }
    return true;
}

// 4 consecutive fp32 values split into the hi / lo tiles at byte offset off.
__device__ __forceinline__ void ta_store4(uint8_t* hi, uint8_t* lo, uint32_t off, float4 v) {
    float4 h, l;
    tc::split_tf32(v.x, h.x, l.x);
    tc::split_tf32(v.y, h.y, l.y);
    tc::split_tf32(v.z, h.z, l.z);
    tc::split_tf32(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
}

template <int HD, int GROUP>
__global__ void __launch_bounds__(TA_THREADS, 1)
k_pf_attn_tc(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
             float* __restrict__ out, int T, int pos0, int nh, int max_seq, unsigned* err) {
    using L = TaLayout<HD>;
    constexpr int BQ = TA_R / GROUP;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[9];
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // grid (KV heads, query blocks), heads fastest: CTAs start in order of
    // decreasing length (the longest query blocks of every head first)
    const int g = blockIdx.x;
    const int qb = gridDim.y - 1 - blockIdx.y;
    const int q0 = qb * BQ, QD = nh * HD;
    const float* kh = kc + (size_t)g * max_seq * HD;
    const float* vh = vc + (size_t)g * max_seq * HD;
    const int kend = pos0 + min(q0 + BQ, T);     // keys 0 .. kend - 1
    const int nt = (kend + TA_NK - 1) / TA_NK;
    const uint32_t b0 = tc::smem_u32(&bars[0]);
    const uint32_t kfull = b0, kempty = b0 + 8, vfull = b0 + 16, pfull = b0 + 24, pvdone = b0 + 32;
    const uint32_t sfull = b0 + 40, sfree = b0 + 56;   // [2] each
    if (tid == 0) {
        mbs_init(kfull, 4);    // the converter warps
        mbs_init(kempty, 1);   // MMA commit: the scores of the K tile are done
        mbs_init(vfull, 4);
        mbs_init(pfull, 4);    // the softmax warps: P written, O rescaled
        mbs_init(pvdone, 1);   // MMA commit: O += P V done
        for (int b = 0; b < 2; b++) {
            mbs_init(sfull + 8 * b, 1);
            mbs_init(sfree + 8 * b, 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) tc::tmem_alloc(&tmem_slot, L::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    if (warp < 4) {   // Q row r (head g GROUP + r / BQ, query q0 + r % BQ; zero past T) into tensor-memory lane r
        const int r = tid, t = q0 + r % BQ, h = g * GROUP + r / BQ;
        const float* src = q + (size_t)t * QD + (size_t)h * HD;
        const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
            float hv[16], lv[16];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < T) v = __ldg(reinterpret_cast<const float4*>(src + c + i));
                tc::split_tf32(v.x, hv[i], lv[i]);
                tc::split_tf32(v.y, hv[i + 1], lv[i + 1]);
                tc::split_tf32(v.z, hv[i + 2], lv[i + 2]);
                tc::split_tf32(v.w, hv[i + 3], lv[i + 3]);
            }
            tc::tmem_st16(lb + L::QHI + (uint32_t)c, hv);
            tc::tmem_st16(lb + L::QLO + (uint32_t)c, lv);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    bool ok = true;

    if (warp == 8) {   // ---- MMA issue (one lane)
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_tf32(TA_R, TA_NK), idO = tc::idesc_tf32(TA_R, HD);
            constexpr uint32_t LK = TA_NK / 8 * 128, LP = TA_R / 8 * 128, LV = HD / 8 * 128;
            const uint32_t base = tc::smem_u32(sm);
            auto scores = [&](int t) {   // S[t & 1] = Q K^T: hd / 8 k-steps x 3 products, A from tensor memory
                const uint32_t S = tmem + L::S0 + (uint32_t)(TA_NK * (t & 1));
#pragma unroll
                for (int ks = 0; ks < HD / 8; ks++) {
                    const uint32_t koff = (ks >> 2) * L::KSUB + (ks & 3) * 2 * LK;
                    const uint64_t khd = tc::smem_desc(base + L::K_HI + koff, LK, 128);
                    const uint64_t kld = tc::smem_desc(base + L::K_LO + koff, LK, 128);
                    const uint32_t qh = tmem + L::QHI + (uint32_t)(8 * ks), ql = tmem + L::QLO + (uint32_t)(8 * ks);
                    tc::mma_tf32_ta(S, qh, khd, idS, ks > 0);
                    tc::mma_tf32_ta(S, qh, kld, idS, true);
                    tc::mma_tf32_ta(S, ql, khd, idS, true);
                }
                tc::mma_commit(sfull + 8 * (t & 1));
                tc::mma_commit(kempty);
            };
            if (ok) ok = ta_wait(kfull, 0, err);
            if (ok) {
                tc::fence_after_sync();
                scores(0);
            }
            for (int t = 0; t < nt && ok; t++) {
                if (t + 1 < nt) {   // the next tile's scores run during this tile's softmax
                    ok = ta_wait(kfull, (t + 1) & 1, err);
                    if (ok && t + 1 >= 2) ok = ta_wait(sfree + 8 * ((t + 1) & 1), (((t + 1) >> 1) - 1) & 1, err);
                    if (!ok) break;
                    tc::fence_after_sync();
                    scores(t + 1);
                }
                ok = ta_wait(pfull, t & 1, err) && ta_wait(vfull, t & 1, err);
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t O = tmem + L::OC;
#pragma unroll
                for (int ks = 0; ks < TA_NK / 8; ks++) {   // O (+)= P V over the tile's 64 keys
                    const uint32_t poff = (ks >> 2) * L::PSUB + (ks & 3) * 2 * LP;
                    const uint32_t voff = (ks >> 2) * L::VSUB + (ks & 3) * 2 * LV;
                    const uint64_t ph = tc::smem_desc(base + L::P_HI + poff, LP, 128);
                    const uint64_t pl = tc::smem_desc(base + L::P_LO + poff, LP, 128);
                    const uint64_t vhd = tc::smem_desc(base + L::V_HI + voff, LV, 128);
                    const uint64_t vld = tc::smem_desc(base + L::V_LO + voff, LV, 128);
                    tc::mma_tf32(O, ph, vhd, idO, t > 0 || ks > 0);
                    tc::mma_tf32(O, ph, vld, idO, true);
                    tc::mma_tf32(O, pl, vhd, idO, true);
                }
                tc::mma_commit(pvdone);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {   // ---- warps 4-7: K and V tiles (the next tile's loads issued once this one is stored)
        const int cw = warp - 4, ct = tid - 128;
        // K: lane (j = lane % 8, e = lane / 8) takes keys 8 cw + j and
        // 32 + 8 cw + j, float4 columns 4 it + e of each: a quarter-warp
        // writes one core matrix (8 keys, conflict-free) and reads 8 rows x
        // 16 bytes
        constexpr int KIT = HD / 16;
        const int kj = 8 * cw + (lane & 7), ke = lane >> 3;
        // V^T: thread ct takes head_dim column d = ct % HD and keys kv0 ..
        // kv0 + VK - 1; a warp reads 32 consecutive floats of one key row
        constexpr int VK = TA_NK * HD / 128;   // keys per thread (64 at hd 128, 32 at 64)
        const int vd = ct % HD, kv0 = VK * (ct / HD);
        float4 kr[2][KIT];
        float vr[VK];
        auto load_k = [&](int t) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int key = t * TA_NK + 32 * hh + kj;
#pragma unroll
                for (int i = 0; i < KIT; i++)
                    kr[hh][i] = key < kend
                                    ? __ldg(reinterpret_cast<const float4*>(kh + (size_t)key * HD + 4 * (4 * i + ke)))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        auto load_v = [&](int t) {
#pragma unroll
            for (int i = 0; i < VK; i++) {
                const int kv = t * TA_NK + kv0 + i;
                vr[i] = kv < kend ? __ldg(vh + (size_t)kv * HD + vd) : 0.f;   // rows past the range: zero
            }
        };
        load_k(0);
        load_v(0);
        for (int t = 0; t < nt; t++) {
            // K(t) once the scores of tile t - 1 are done; then tile t + 1's K loads
            if (t > 0 && ok) ok = ta_wait(kempty, (t - 1) & 1, err);
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
#pragma unroll
                for (int i = 0; i < KIT; i++) {
                    const int d = 4 * (4 * i + ke);
                    ta_store4(sm + L::K_HI, sm + L::K_LO,
                              (d >> 5) * L::KSUB + tc::tile_off(32 * hh + kj, d & 31, TA_NK), kr[hh][i]);
                }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) mbs_arrive(kfull);
            if (t + 1 < nt) load_k(t + 1);
            // V(t) once O += P V of tile t - 1 is done; then tile t + 1's V loads
            if (t > 0 && ok) ok = ta_wait(pvdone, (t - 1) & 1, err);
#pragma unroll
            for (int i = 0; i < VK; i += 4) {
                const int key = kv0 + i;
                ta_store4(sm + L::V_HI, sm + L::V_LO, (key >> 5) * L::VSUB + tc::tile_off(vd, key & 31, HD),
                          make_float4(vr[i], vr[i + 1], vr[i + 2], vr[i + 3]));
            }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) mbs_arrive(vfull);
            if (t + 1 < nt) load_v(t + 1);
        }
    } else {   // ---- warps 0-3: softmax, O rescale, output; thread = row r = tensor-memory lane
        const int r = tid;
        const int tq = q0 + r % BQ, h = g * GROUP + r / BQ;
        const int qpos = pos0 + tq;
        const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
        const uint32_t O = lb + L::OC;
        const float scale = 1.0f / sqrtf((float)HD);
        float m = -INFINITY, l = 0.f;
        for (int t = 0; t < nt; t++) {
            const int b = t & 1;
            if (ok) ok = ta_wait(sfull + 8 * b, (t >> 1) & 1, err);
            tc::fence_after_sync();
            float sc[TA_NK];
#pragma unroll
            for (int c = 0; c < TA_NK; c += 16) {
                float a16[16];
                tc::tmem_ld16(lb + L::S0 + (uint32_t)(TA_NK * b + c), a16);
#pragma unroll
                for (int i = 0; i < 16; i++) sc[c + i] = a16[i];
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbs_arrive(sfree + 8 * b);   // S[b] may be overwritten
            // scale, causal mask (key > query position: -inf), online softmax
            // with a lazily updated max: p = exp(s - m) for the row's max m as
            // of its last rescale, which moves (and O, l are rescaled) only
            // when a score exceeds it by more than TA_TAU -- so p <= e^TA_TAU
            // and the rescale of O in tensor memory is rare; O / l is the
            // same softmax for any common m
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < TA_NK; i++) {
                const int key = t * TA_NK + i;
                sc[i] = key > qpos ? -INFINITY : sc[i] * scale;
                mx = fmaxf(mx, sc[i]);
            }
            const bool move = mx > m + TA_TAU;   // always on the first tile (m = -inf; key 0 is in range)
            const float mn = move ? mx : m;
            const float alpha = expf(m - mn);    // 1 when the max stays, 0 on the first tile
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < TA_NK; i++) {
                sc[i] = expf(sc[i] - mn);
                sum += sc[i];
            }
            l = fmaf(l, alpha, sum);
            m = mn;
            if (t > 0) {   // P and V of tile t - 1 consumed, O holds its sum: rescale O if a row's max moved
                if (ok) ok = ta_wait(pvdone, (t - 1) & 1, err);
                tc::fence_after_sync();
                if (__any_sync(0xffffffffu, move)) {
#pragma unroll 1
                    for (int c = 0; c < HD; c += 16) {
                        float o16[16];
                        tc::tmem_ld16(O + (uint32_t)c, o16);
#pragma unroll
                        for (int i = 0; i < 16; i++) o16[i] *= alpha;
                        tc::tmem_st16(O + (uint32_t)c, o16);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < TA_NK / 4; j++)
                ta_store4(sm + L::P_HI, sm + L::P_LO, (j >> 3) * L::PSUB + tc::tile_off(r, 4 * (j & 7), TA_R),
                          make_float4(sc[4 * j], sc[4 * j + 1], sc[4 * j + 2], sc[4 * j + 3]));
            tc::fence_async_smem();   // P (generic stores) -> tensor-core reads
            tc::fence_before_sync();  // O (tensor-memory stores) -> the next MMA
            __syncwarp();
            if (lane == 0) mbs_arrive(pfull);
        }
        if (ok) ok = ta_wait(pvdone, (nt - 1) & 1, err);
        tc::fence_after_sync();
        const float inv = 1.0f / l;
        float* dst = out + (size_t)tq * QD + (size_t)h * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
            float o16[16];
            tc::tmem_ld16(O + (uint32_t)c, o16);
            if (tq < T && ok)
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<float4*>(dst + c + i) =
                        make_float4(o16[i] * inv, o16[i + 1] * inv, o16[i + 2] * inv, o16[i + 3] * inv);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 8) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

template <int HD, int GROUP>
static cudaError_t launch_pf_attn_tc(const float* q, const float* kc, const float* vc, float* out, int T, int pos0,
                                     int n_kv, int max_seq, unsigned* err, cudaStream_t st) {
    constexpr int smem = TaLayout<HD>::SMEM;
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(k_pf_attn_tc<HD, GROUP>), smem);
    if (e != cudaSuccess) return e;
    constexpr int BQ = TA_R / GROUP;
    if ((T + BQ - 1) / BQ > 65535) return cudaErrorInvalidValue;   // grid.y limit: 2M prompt rows at GROUP 4
    dim3 grid(n_kv, (T + BQ - 1) / BQ);
    k_pf_attn_tc<HD, GROUP><<<grid, TA_THREADS, smem, st>>>(q, kc, vc, out, T, pos0, n_kv * GROUP, max_seq, err);
    return cudaGetLastError();
}

// GB_PF_ATTN=cuda selects the CUDA-core kernel (for comparison); the default
// is the tensor-core kernel.
static bool pf_attn_tensor_cores() {
    static const bool tc = [] {
        const char* e = getenv("GB_PF_ATTN");
        return !(e && !strcmp(e, "cuda"));
    }();
    return tc;
}

int prefill_attention(const float* q, const float* kc, const float* vc, float* out, int T, int pos0, int n_heads,
                      int n_kv, int head_dim, int max_seq, cudaStream_t st, unsigned* err) {
    if (!q || !kc || !vc || !out || T <= 0 || pos0 < 0 || n_kv <= 0 || n_heads % n_kv || pos0 + T > max_seq)
        return GB_EINVAL;
    if (!err) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_pf_err) != cudaSuccess) return GB_ECUDA;
        err = static_cast<unsigned*>(p);
    }
    const int group = n_heads / n_kv;
    const bool tcore = pf_attn_tensor_cores();
    cudaError_t e = cudaErrorInvalidValue;
#define GB_PA_CASE(HDV, GV)                                                                            \
    if (head_dim == HDV && group == GV)                                                                \
        e = tcore ? launch_pf_attn_tc<HDV, GV>(q, kc, vc, out, T, pos0, n_kv, max_seq, err, st)        \
                  : launch_pf_attn<HDV, GV>(q, kc, vc, out, T, pos0, n_kv, max_seq, st);
    GB_PA_CASE(128, 1) GB_PA_CASE(128, 2) GB_PA_CASE(128, 4) GB_PA_CASE(128, 8)
    GB_PA_CASE(64, 1) GB_PA_CASE(64, 2) GB_PA_CASE(64, 4) GB_PA_CASE(64, 8)
#undef GB_PA_CASE
    if (e == cudaErrorInvalidValue) return GB_EINVAL;
    return e == cudaSuccess ? GB_OK : GB_ECUDA;
}

// ---------------------------------------------------------------- one layer
int enqueue_prefill_layer(const PrefillArgs& a, cudaStream_t st) {
    const int T = a.T, H = a.H, QD = a.n_heads * a.hd, KVD = a.n_kv * a.hd, F = a.ff;
    int rc;
    // fp16 operands: each GEMM input split once (shared by q / k / v and
    // by gate / up)
    const bool f16 = gemm_f16_operands();
    const GemmX16 x16{a.xh, a.xl, a.xinv, gemm_split_rows(T)};
    auto split = [&](const float* x, int K) { return f16 ? gemm_split_x(x, T, K, a.xh, a.xl, a.xinv, st) : GB_OK; };
    const GemmX16* xm = f16 ? &x16 : nullptr;
    auto gemm_on = [&](cudaStream_t s, int which, const float* x, float* y, const float* res, int N, int K) {
        return gemm_launch(a.dt[which], a.w[which], x, y, res, N, K, T, s, a.err, 0, xm);
    };
    auto gemm = [&](int which, const float* x, float* y, const float* res, int N, int K) {
        return gemm_on(st, which, x, y, res, N, K);
    };
    // RMSNorm: with fp16 operands straight into the split (xn not written)
    auto norm = [&](const float* w) {
        return f16 ? gemm_rmsnorm_split_x(a.hidden, w, T, H, a.eps, a.xh, a.xl, a.xinv, st)
                   : rmsnorm_rows(a.hidden, w, a.xn, H, T, a.eps, st);
    };
    if ((rc = norm(a.ra))) return rc;
    // wk and wv (few CTAs each) on the side stream beside wq, whose last wave
    // leaves most SMs idle; all three only read the split of xn
    cudaStream_t kv = a.side ? a.side : st;
    if (a.side) {
        if (cudaEventRecord(a.fork, st) != cudaSuccess || cudaStreamWaitEvent(a.side, a.fork, 0) != cudaSuccess)
            return GB_ECUDA;
    }
    if ((rc = gemm(GB_WQ, a.xn, a.q, nullptr, QD, H))) return rc;
    if ((rc = gemm_on(kv, GB_WK, a.xn, a.k, nullptr, KVD, H))) return rc;
    if ((rc = gemm_on(kv, GB_WV, a.xn, a.v, nullptr, KVD, H))) return rc;
    if (a.side) {
        if (cudaEventRecord(a.join, a.side) != cudaSuccess || cudaStreamWaitEvent(st, a.join, 0) != cudaSuccess)
            return GB_ECUDA;
    }
    k_pf_rope_kv<<<T, 256, 0, st>>>(a.q, a.k, a.v, a.kc, a.vc, a.rope, a.pos0, a.n_heads, a.n_kv, a.hd, a.max_seq);
    if (cudaGetLastError() != cudaSuccess) return GB_ECUDA;
    if ((rc = prefill_attention(a.q, a.kc, a.vc, a.attn, T, a.pos0, a.n_heads, a.n_kv, a.hd, a.max_seq, st, a.err)))
        return rc;
    if ((rc = split(a.attn, QD))) return rc;
    if ((rc = gemm(GB_WO, a.attn, a.hidden, a.hidden, H, QD))) return rc;
    if ((rc = norm(a.rf))) return rc;
    // gate / up rows are fk wide (ffn_down's columns); columns F .. fk - 1
    // stay zero (the prefill buffer is zeroed once and never written there)
    const int FK = a.fk;
    if (a.dt[GB_WGATE] == a.dt[GB_WUP]) {   // silu(gate) * up straight from one GEMM
        if ((rc = gemm_swiglu_launch(a.dt[GB_WGATE], a.w[GB_WGATE], a.w[GB_WUP], a.xn, a.gate, F, H, T, st, a.err, FK,
                                     xm)))
            return rc;
    } else {
        if ((rc = gemm_launch(a.dt[GB_WGATE], a.w[GB_WGATE], a.xn, a.gate, nullptr, F, H, T, st, a.err, FK, xm)))
            return rc;
        if ((rc = gemm_launch(a.dt[GB_WUP], a.w[GB_WUP], a.xn, a.up, nullptr, F, H, T, st, a.err, FK, xm))) return rc;
        if ((rc = gb_silu_mul(a.gate, a.up, T * FK, st))) return rc;   // silu(0) * 0 = 0 in the padding
    }
    if ((rc = split(a.gate, FK))) return rc;
    return gemm(GB_WDOWN, a.gate, a.hidden, a.hidden, H, FK);
}

}  // namespace gb

extern "C" int gb_prefill_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                                    int n_tokens, int pos, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                    void* stream) {
    return gb::prefill_attention(q, k_cache, v_cache, out, n_tokens, pos, n_heads, n_kv_heads, head_dim, max_seq,
                                 static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int gb_prefill_attention_error(int clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, gb::g_pf_err, sizeof(v)) != cudaSuccess) return GB_ECUDA;
    if (clear && v) {
        const unsigned z = 0;
        if (cudaMemcpyToSymbol(gb::g_pf_err, &z, sizeof(z)) != cudaSuccess) return GB_ECUDA;
    }
    return -(int)v;
}
