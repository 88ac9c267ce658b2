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
//   xn = RMSNorm(h); gate, up       k_rmsnorm, gb_gemm x 2
//   gate = silu(gate) * up          k_silu_mul
//   h += gate . Wdown^T             gb_gemm with the residual
//
// Activations are row-major [T][width] fp32 in HBM; the K / V caches keep the
// decode layout [n_kv][max_seq][hd], so decode continues from pos0 + T.
#include "gb_common.cuh"
#include "gb_internal.h"

namespace gb {

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

int prefill_attention(const float* q, const float* kc, const float* vc, float* out, int T, int pos0, int n_heads,
                      int n_kv, int head_dim, int max_seq, cudaStream_t st) {
    if (!q || !kc || !vc || !out || T <= 0 || pos0 < 0 || n_kv <= 0 || n_heads % n_kv || pos0 + T > max_seq)
        return GB_EINVAL;
    const int group = n_heads / n_kv;
    cudaError_t e = cudaErrorInvalidValue;
#define GB_PA_CASE(HDV, GV) \
    if (head_dim == HDV && group == GV) e = launch_pf_attn<HDV, GV>(q, kc, vc, out, T, pos0, n_kv, max_seq, st);
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
    auto gemm = [&](int which, const float* x, float* y, const float* res, int N, int K) {
        return gemm_launch(a.dt[which], a.w[which], x, y, res, N, K, T, st, a.err);
    };
    if ((rc = rmsnorm_rows(a.hidden, a.ra, a.xn, H, T, a.eps, st))) return rc;
    if ((rc = gemm(GB_WQ, a.xn, a.q, nullptr, QD, H))) return rc;
    if ((rc = gemm(GB_WK, a.xn, a.k, nullptr, KVD, H))) return rc;
    if ((rc = gemm(GB_WV, a.xn, a.v, nullptr, KVD, H))) return rc;
    k_pf_rope_kv<<<T, 256, 0, st>>>(a.q, a.k, a.v, a.kc, a.vc, a.rope, a.pos0, a.n_heads, a.n_kv, a.hd, a.max_seq);
    if (cudaGetLastError() != cudaSuccess) return GB_ECUDA;
    if ((rc = prefill_attention(a.q, a.kc, a.vc, a.attn, T, a.pos0, a.n_heads, a.n_kv, a.hd, a.max_seq, st)))
        return rc;
    if ((rc = gemm(GB_WO, a.attn, a.hidden, a.hidden, H, QD))) return rc;
    if ((rc = rmsnorm_rows(a.hidden, a.rf, a.xn, H, T, a.eps, st))) return rc;
    if ((rc = gemm(GB_WGATE, a.xn, a.gate, nullptr, F, H))) return rc;
    if ((rc = gemm(GB_WUP, a.xn, a.up, nullptr, F, H))) return rc;
    if ((rc = gb_silu_mul(a.gate, a.up, T * F, st))) return rc;
    return gemm(GB_WDOWN, a.gate, a.hidden, a.hidden, H, F);
}

}  // namespace gb

extern "C" int gb_prefill_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                                    int n_tokens, int pos, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                    void* stream) {
    return gb::prefill_attention(q, k_cache, v_cache, out, n_tokens, pos, n_heads, n_kv_heads, head_dim, max_seq,
                                 static_cast<cudaStream_t>(stream));
}
