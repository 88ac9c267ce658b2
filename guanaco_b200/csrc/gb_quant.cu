// gb_quant.cu -- fused dequantise + matvec over GGUF Q4_K / Q6_K / Q8_0 blocks,
// bit-exact dequantisers, and the seeded synthetic block generators.
//
// Reference semantics: y[r] = sum_c dequant(W[r, c]) * x[c]
//   Q4_K  src/kernels/cpu/quant_matvec_q4_k.c:65-173 (w = d*sc*q - dmin*m)
//   Q6_K  src/kernels/cpu/quant_matvec_q6_k.c:43-98  (w = d*sc*(q - 32))
//   Q8_0  src/kernels/cpu/quant_matvec_q8_0.c:41-78  (w = d*q)
// The reference CUDA kernels these replace are matvec_q4k_kernel
// (src/kernels/cuda/matvec_q4k_cuda.cu:29-77) and matvec_q6k_kernel
// (src/kernels/cuda/cuda_layer_kernels.cu:26-75); there was no Q8_0 kernel.
//
// Kernel shape (batch-1 GEMV, HBM-bound, CUDA cores only):
//   * weights stream straight from HBM into registers with 128-bit (Q4_K,
//     always 16-byte aligned) or aligned 32-bit windows + funnel shifts (Q6_K
//     210-byte and Q8_0 34-byte blocks are only 2-byte aligned);
//   * each CTA stages x once in shared memory, already multiplied by the
//     per-position power of two that the in-place field extraction needs
//     (see gb::lin) and swizzled so the 128-bit reads are bank-conflict free,
//     together with per-lane partial sums of x for the min / -32 / +128 terms;
//   * a warp owns R rows and a slice of the column chunks (the CTA's 8 warps
//     are WR row groups x WK column slices), so every x value read from shared
//     memory feeds R rows;
//   * partial sums reduce with warp shuffles, then across the WK slices in
//     shared memory; the epilogue optionally adds a residual vector.
#include "gb_common.cuh"
#include "gb_internal.h"

namespace gb {

constexpr float P100 = 0x1p100f, P96 = 0x1p96f, P92 = 0x1p92f, P88 = 0x1p88f;
constexpr float P84 = 0x1p84f, P80 = 0x1p80f, P49 = 0x1p49f;

// 8 bytes starting at a 2-byte-aligned address, from two aligned words, one
// aligned half word and two funnel shifts.  The shift is 0 or 16, so only the
// low half of the third piece is ever used and the window never reads past
// p + 8 (blocks at the very end of a matrix stay in bounds).
struct Pair32 { uint32_t lo, hi; };
__device__ __forceinline__ Pair32 load8_unaligned(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1), w2 = ldg_u16(w + 2);
    return {__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh)};
}

// ------------------------------------------------------------------ Q4_K
// Lane map per warp chunk of 4 blocks: block = lane>>3, segment s = lane&7
// covers qs bytes [16s, 16s+16): pair i = s>>1 (sub-blocks 2i lo nibble,
// 2i+1 hi nibble), half h = s&1 -> 16 weights of each sub-block.
struct FQ4K {
    static constexpr int CB = 4;        // blocks per chunk
    static constexpr int BW = 256;      // weights per block
    static constexpr int BYTES = GB_Q4K_BYTES;
    static constexpr int SLOTS = 8;     // float4 x slots per lane
    struct Regs { uint4 h, q; };

    __device__ static int block_of(int c, int lane) { return c * CB + (lane >> 3); }

    // x slot k of lane L: k>>2 selects lo/hi sub-block, k&3 the qs word.
    __device__ static float4 stage(const float* x, int b, int L, int k) {
        const int s = L & 7, i = s >> 1, h = s & 1, hi = k >> 2, t = k & 3;
        const float4 v = *reinterpret_cast<const float4*>(x + b * 256 + 64 * i + 32 * hi + 16 * h + 4 * t);
        return hi ? make_float4(v.x * P96, v.y * P88, v.z * P80, v.w * P80)
                  : make_float4(v.x * P100, v.y * P92, v.z * P84, v.w * P84);
    }
    // (sum of x over this lane's 16 lo columns, same for hi, 0, 0)
    __device__ static float4 stage_sx(const float* x, int b, int L) {
        const int s = L & 7, i = s >> 1, h = s & 1;
        float r[2];
#pragma unroll
        for (int hi = 0; hi < 2; hi++) {
            const float4* p = reinterpret_cast<const float4*>(x + b * 256 + 64 * i + 32 * hi + 16 * h);
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) { const float4 v = p[k]; acc += (v.x + v.y) + (v.z + v.w); }
            r[hi] = acc;
        }
        return make_float4(r[0], r[1], 0.f, 0.f);
    }
    __device__ static void load(const uint8_t* blk, int lane, Regs& r) {
        r.h = ldg4_stream(blk);
        r.q = ldg4_stream(blk + 16 + 16 * (lane & 7));
    }
    __device__ static float dot(const Regs& r, const float4* xs, float4 sx, int lane) {
        const int pair = (lane & 7) >> 1;
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&r.h.x));
        uint32_t scw, mw;
        if (pair < 2) {
            scw = r.h.y & 0x3F3F3F3Fu;
            mw = r.h.z & 0x3F3F3F3Fu;
        } else {
            scw = (r.h.w & 0x0F0F0F0Fu) | ((r.h.y >> 2) & 0x30303030u);
            mw = ((r.h.w >> 4) & 0x0F0F0F0Fu) | ((r.h.z >> 2) & 0x30303030u);
        }
        const int sh = (pair & 1) << 4;
        const float sa = (float)((scw >> sh) & 0xFFu), sb = (float)((scw >> (sh + 8)) & 0xFFu);
        const float ma = (float)((mw >> sh) & 0xFFu), mb = (float)((mw >> (sh + 8)) & 0xFFu);
        float2 alo = make_float2(0.f, 0.f), ahi = make_float2(0.f, 0.f);
        const uint32_t qw[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t w = qw[t], w8 = w >> 8;
            const float4 xl = xs[t], xh = xs[4 + t];
            alo = ffma2(make_float2(lin(w & 0xFu), lin(w & 0xF00u)), make_float2(xl.x, xl.y), alo);
            alo = ffma2(make_float2(lin(w & 0xF0000u), lin(w8 & 0xF0000u)), make_float2(xl.z, xl.w), alo);
            ahi = ffma2(make_float2(lin(w & 0xF0u), lin(w & 0xF000u)), make_float2(xh.x, xh.y), ahi);
            ahi = ffma2(make_float2(lin(w & 0xF00000u), lin(w8 & 0xF00000u)), make_float2(xh.z, xh.w), ahi);
        }
        const float d49 = dm.x * P49;
        return d49 * (sa * (alo.x + alo.y) + sb * (ahi.x + ahi.y)) - dm.y * (ma * sx.x + mb * sx.y);
    }
};

// ------------------------------------------------------------------ Q6_K
// Lane map per chunk of 4 blocks: block = lane>>3, s = lane&7: half n = s>>2,
// l0 = (s&3)*8 -> weights l, l+32, l+64, l+96 (groups G = 0..3) for
// l in [l0, l0+8) of half n: 32 weights, scales sc[8n + l0/16 + 2G].
struct FQ6K {
    static constexpr int CB = 4;
    static constexpr int BW = 256;
    static constexpr int BYTES = GB_Q6K_BYTES;
    static constexpr int SLOTS = 8;
    struct Regs { uint32_t a0, a1, b0, b1, h0, h1, sc, d; };

    __device__ static int block_of(int c, int lane) { return c * CB + (lane >> 3); }

    // slot k: group G = k>>1, word t = k&1 -> columns l0 + 4t + [0,4).
    __device__ static float4 stage(const float* x, int b, int L, int k) {
        const int s = L & 7, n = s >> 2, l0 = (s & 3) * 8, G = k >> 1, t = k & 1;
        const float4 v = *reinterpret_cast<const float4*>(x + b * 256 + 128 * n + 32 * G + l0 + 4 * t);
        return make_float4(v.x * P100, v.y * P92, v.z * P84, v.w * P84);
    }
    // 32 * (sum of x over the lane's 8 columns of group G), G = 0..3.
    __device__ static float4 stage_sx(const float* x, int b, int L) {
        const int s = L & 7, n = s >> 2, l0 = (s & 3) * 8;
        float r[4];
#pragma unroll
        for (int G = 0; G < 4; G++) {
            const float4* p = reinterpret_cast<const float4*>(x + b * 256 + 128 * n + 32 * G + l0);
            const float4 u = p[0], v = p[1];
            r[G] = 32.f * (((u.x + u.y) + (u.z + u.w)) + ((v.x + v.y) + (v.z + v.w)));
        }
        return make_float4(r[0], r[1], r[2], r[3]);
    }
    __device__ static void load(const uint8_t* blk, int lane, Regs& r) {
        const int s = lane & 7, n = s >> 2, l0 = (s & 3) * 8, is = (s & 3) >> 1;
        const Pair32 a = load8_unaligned(blk + 64 * n + l0);
        const Pair32 b = load8_unaligned(blk + 64 * n + 32 + l0);
        const Pair32 h = load8_unaligned(blk + 128 + 32 * n + l0);
        r.a0 = a.lo; r.a1 = a.hi; r.b0 = b.lo; r.b1 = b.hi; r.h0 = h.lo; r.h1 = h.hi;
        const uint8_t* sp = blk + 192 + 8 * n + is;
        r.sc = (uint32_t)__ldg(sp) | ((uint32_t)__ldg(sp + 2) << 8) |
               ((uint32_t)__ldg(sp + 4) << 16) | ((uint32_t)__ldg(sp + 6) << 24);
        r.d = ldg_u16(blk + 208);
    }
    __device__ static float dot(const Regs& r, const float4* xs, float4 sx, int) {
        float2 acc[4];
#pragma unroll
        for (int G = 0; G < 4; G++) acc[G] = make_float2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 2; t++) {
            const uint32_t a = t ? r.a1 : r.a0, b = t ? r.b1 : r.b0, h = t ? r.h1 : r.h0;
            uint32_t g[4];
            g[0] = (a & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
            g[1] = (b & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
            g[2] = ((a >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);
            g[3] = ((b >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
#pragma unroll
            for (int G = 0; G < 4; G++) {
                const float4 xv = xs[2 * G + t];
                acc[G] = ffma2(make_float2(lin(g[G] & 0x3Fu), lin(g[G] & 0x3F00u)), make_float2(xv.x, xv.y), acc[G]);
                acc[G] = ffma2(make_float2(lin(g[G] & 0x3F0000u), lin(b3_to_b2(g[G]))), make_float2(xv.z, xv.w), acc[G]);
            }
        }
        const float sxg[4] = {sx.x, sx.y, sx.z, sx.w};
        float tot = 0.f;
#pragma unroll
        for (int G = 0; G < 4; G++) {
            const float scg = (float)(int)(int8_t)(r.sc >> (8 * G));
            tot += scg * fmaf(acc[G].x + acc[G].y, P49, -sxg[G]);
        }
        return __half2float(__ushort_as_half((unsigned short)r.d)) * tot;
    }
};

// ------------------------------------------------------------------ Q8_0
// Lane map per chunk of 8 blocks: block = lane>>2, s = lane&3 -> quants
// [8s, 8s+8).  Quants are read as unsigned bytes u = q + 128 (XOR 0x80).
struct FQ80 {
    static constexpr int CB = 8;
    static constexpr int BW = 32;
    static constexpr int BYTES = GB_Q80_BYTES;
    static constexpr int SLOTS = 2;
    struct Regs { uint32_t w0, w1, d; };

    __device__ static int block_of(int c, int lane) { return c * CB + (lane >> 2); }
    __device__ static float4 stage(const float* x, int b, int L, int k) {
        const float4 v = *reinterpret_cast<const float4*>(x + b * 32 + 8 * (L & 3) + 4 * k);
        return make_float4(v.x * P100, v.y * P92, v.z * P84, v.w * P84);
    }
    __device__ static float4 stage_sx(const float* x, int b, int L) {
        const float4* p = reinterpret_cast<const float4*>(x + b * 32 + 8 * (L & 3));
        const float4 u = p[0], v = p[1];
        return make_float4(128.f * (((u.x + u.y) + (u.z + u.w)) + ((v.x + v.y) + (v.z + v.w))), 0.f, 0.f, 0.f);
    }
    __device__ static void load(const uint8_t* blk, int lane, Regs& r) {
        const Pair32 q = load8_unaligned(blk + 2 + 8 * (lane & 3));
        r.w0 = q.lo; r.w1 = q.hi;
        r.d = ldg_u16(blk);
    }
    __device__ static float dot(const Regs& r, const float4* xs, float4 sx, int) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 2; t++) {
            const uint32_t u = (t ? r.w1 : r.w0) ^ 0x80808080u;
            const float4 xv = xs[t];
            acc = ffma2(make_float2(lin(u & 0xFFu), lin(u & 0xFF00u)), make_float2(xv.x, xv.y), acc);
            acc = ffma2(make_float2(lin(u & 0xFF0000u), lin(b3_to_b2(u))), make_float2(xv.z, xv.w), acc);
        }
        return __half2float(__ushort_as_half((unsigned short)r.d)) * fmaf(acc.x + acc.y, P49, -sx.x);
    }
};

template <int SLOTS>
__device__ __forceinline__ int swz(int L, int k) {
    if constexpr (SLOTS == 8) return k ^ (L & 7);
    else return k ^ ((L >> 2) & 1);
}

// Shared-memory bytes the kernel needs for nb blocks per row.
template <class F>
__host__ __device__ constexpr size_t smem_bytes(int nb) {
    return (size_t)((nb + F::CB - 1) / F::CB) * 32 * (F::SLOTS + 1) * sizeof(float4) + 8 * 4 * sizeof(float) * 8;
}

// y[r] = W[r,:] . x (+ residual[r]).  R rows per warp; the 8 warps are
// (8 >> wk_log2) row groups x (1 << wk_log2) column slices.  Persistent over
// row tiles.  x must hold nb * F::BW floats, 16-byte aligned.
template <class F, int R>
__global__ void __launch_bounds__(256, 2)
k_matvec(const uint8_t* __restrict__ W, int rows, int nb, const float* __restrict__ x,
         float* __restrict__ y, const float* __restrict__ residual, int wk_log2) {
    extern __shared__ float4 smem[];
    const int nchunks = (nb + F::CB - 1) / F::CB;
    float4* xs = smem;
    float4* sxs = smem + (size_t)nchunks * 32 * F::SLOTS;
    float* red = reinterpret_cast<float*>(sxs + (size_t)nchunks * 32);   // [WK][WR*R]
    const int tid = threadIdx.x;

    // ---- stage prescaled x and per-lane x sums (blocks past nb stage zeros)
    for (int e = tid; e < nchunks * 32 * F::SLOTS; e += blockDim.x) {
        const int c = e / (32 * F::SLOTS), L = (e / F::SLOTS) & 31, k = e % F::SLOTS;
        const int b = F::block_of(c, L);
        const float4 v = b < nb ? F::stage(x, b, L, k) : make_float4(0.f, 0.f, 0.f, 0.f);
        xs[(size_t)(c * 32 + L) * F::SLOTS + swz<F::SLOTS>(L, k)] = v;
    }
    for (int e = tid; e < nchunks * 32; e += blockDim.x) {
        const int c = e >> 5, L = e & 31, b = F::block_of(c, L);
        sxs[e] = b < nb ? F::stage_sx(x, b, L) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    const int WK = 1 << wk_log2, WR = 8 >> wk_log2;
    const int wr = warp >> wk_log2, wk = warp & (WK - 1);
    const int rows_per_cta = WR * R;
    const size_t row_bytes = (size_t)nb * F::BYTES;

    for (int tile = blockIdx.x; tile * rows_per_cta < rows; tile += gridDim.x) {
        const int row0 = tile * rows_per_cta + wr * R;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.f;

        typename F::Regs cur[R], nxt[R];
        int c = wk;
        if (c < nchunks) {
            const int b = min(F::block_of(c, lane), nb - 1);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = min(row0 + r, rows - 1);
                F::load(W + row * row_bytes + (size_t)b * F::BYTES, lane, cur[r]);
            }
        }
        for (; c < nchunks; c += WK) {
            const int cn = c + WK;
            if (cn < nchunks) {
                const int b = min(F::block_of(cn, lane), nb - 1);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int row = min(row0 + r, rows - 1);
                    F::load(W + row * row_bytes + (size_t)b * F::BYTES, lane, nxt[r]);
                }
            }
            if (F::block_of(c, lane) < nb) {
                float4 xv[F::SLOTS];
#pragma unroll
                for (int k = 0; k < F::SLOTS; k++)
                    xv[k] = xs[(size_t)(c * 32 + lane) * F::SLOTS + swz<F::SLOTS>(lane, k)];
                const float4 sx = sxs[c * 32 + lane];
#pragma unroll
                for (int r = 0; r < R; r++) acc[r] += F::dot(cur[r], xv, sx, lane);
            }
#pragma unroll
            for (int r = 0; r < R; r++) cur[r] = nxt[r];
        }
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);

        if (WK == 1) {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int row = row0 + r;
                    if (row < rows) y[row] = acc[r] + (residual ? residual[row] : 0.f);
                }
            }
        } else {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; r++) red[wk * rows_per_cta + wr * R + r] = acc[r];
            }
            __syncthreads();
            if (tid < rows_per_cta) {
                float s = 0.f;
                for (int k = 0; k < WK; k++) s += red[k * rows_per_cta + tid];
                const int row = tile * rows_per_cta + tid;
                if (row < rows) y[row] = s + (residual ? residual[row] : 0.f);
            }
            __syncthreads();
        }
    }
}

// ------------------------------------------------------------------ launch
template <class F, int R>
static cudaError_t launch_one(const void* W, int rows, int nb, const float* x, float* y,
                              const float* residual, int wk_log2, cudaStream_t st) {
    const size_t smem = smem_bytes<F>(nb);
    static unsigned configured = 0;  // bit per device: shared-memory opt-in done
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(k_matvec<F, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured |= 1u << (dev & 31);
    }
    const int rows_per_cta = (8 >> wk_log2) * R;
    const int tiles = (rows + rows_per_cta - 1) / rows_per_cta;
    const int grid = tiles < 2 * GB_NUM_SMS ? tiles : 2 * GB_NUM_SMS;
    k_matvec<F, R><<<grid, 256, smem, st>>>(static_cast<const uint8_t*>(W), rows, nb, x, y, residual, wk_log2);
    return cudaGetLastError();
}

// Pick rows-per-warp R and the column split WK so the grid covers the GPU.
template <class F>
static cudaError_t launch_fmt(const void* W, int rows, int nb, const float* x, float* y,
                              const float* residual, cudaStream_t st) {
    const int nchunks = (nb + F::CB - 1) / F::CB;
    const int target = 2 * GB_NUM_SMS;
    int bestR = 1, bestK = 0;
    long best_tiles = -1;
    bool found = false;
    for (int R = 4; R >= 1 && !found; R >>= 1) {
        for (int k = 0; k <= 3; k++) {
            if ((1 << k) > nchunks && k > 0) break;
            const long tiles = (rows + (8 >> k) * R - 1) / ((8 >> k) * R);
            if (tiles > best_tiles) { best_tiles = tiles; bestR = R; bestK = k; }
            if (tiles >= target) { bestR = R; bestK = k; found = true; break; }
        }
    }
    if (smem_bytes<F>(nb) > 200 * 1024) return cudaErrorInvalidValue;
    switch (bestR) {
        case 4: return launch_one<F, 4>(W, rows, nb, x, y, residual, bestK, st);
        case 2: return launch_one<F, 2>(W, rows, nb, x, y, residual, bestK, st);
        default: return launch_one<F, 1>(W, rows, nb, x, y, residual, bestK, st);
    }
}

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

__global__ void k_synth_q4k(uint8_t* B, size_t nblocks, uint64_t seed, uint64_t stream) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint8_t* blk = B + b * GB_Q4K_BYTES;
    const uint64_t i0 = (uint64_t)b * 32;
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

__global__ void k_synth_q6k(uint8_t* B, size_t nblocks, uint64_t seed, uint64_t stream) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint8_t* blk = B + b * GB_Q6K_BYTES;    // 2-byte aligned: write 16-bit halves
    uint16_t* d16 = reinterpret_cast<uint16_t*>(blk);
    const uint64_t i0 = (uint64_t)b * 32;
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

__global__ void k_synth_q8_0(uint8_t* B, size_t nblocks, uint64_t seed, uint64_t stream) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint16_t* d16 = reinterpret_cast<uint16_t*>(B + b * GB_Q80_BYTES);
    const uint64_t i0 = (uint64_t)b * 8;
    d16[0] = synth_scale(rand64(seed, stream, i0));
    for (int w = 0; w < 4; w++) {
        const uint64_t r = rand64(seed, stream, i0 + 1 + w);
        for (int k = 0; k < 4; k++) d16[1 + 4 * w + k] = (uint16_t)(r >> (16 * k));
    }
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

extern "C" int gb_matvec(int dtype, const void* W, int rows, int cols, const float* x, float* y,
                         const float* residual, void* stream) {
    if (!W || !x || !y || rows <= 0 || cols <= 0) return GB_EINVAL;
    // Q4_K blocks are read with 128-bit loads (16-byte alignment); Q6_K / Q8_0
    // blocks need 2-byte alignment; x is staged with 128-bit loads.
    const uintptr_t wa = reinterpret_cast<uintptr_t>(W);
    if ((dtype == GB_DT_Q4_K ? (wa & 15) : (wa & 1)) || (reinterpret_cast<uintptr_t>(x) & 15)) return GB_EINVAL;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    switch (dtype) {
        case GB_DT_Q4_K:
            if (cols % 256) return GB_ESHAPE;
            e = launch_fmt<FQ4K>(W, rows, cols / 256, x, y, residual, st);
            break;
        case GB_DT_Q6_K:
            if (cols % 256) return GB_ESHAPE;
            e = launch_fmt<FQ6K>(W, rows, cols / 256, x, y, residual, st);
            break;
        case GB_DT_Q8_0:
            if (cols % 32) return GB_ESHAPE;
            e = launch_fmt<FQ80>(W, rows, cols / 32, x, y, residual, st);
            break;
        default:
            return GB_EINVAL;
    }
    return e == cudaSuccess ? GB_OK : (e == cudaErrorInvalidValue ? GB_ELIMIT : GB_ECUDA);
}

extern "C" int gb_dequant(int dtype, const void* blocks, size_t nblocks, float* out, void* stream) {
    if (!blocks || !out) return GB_EINVAL;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (nblocks == 0) return GB_OK;
    const uint8_t* B = static_cast<const uint8_t*>(blocks);
    switch (dtype) {
        case GB_DT_Q4_K: k_dequant_q4k<<<(unsigned)((nblocks * 128 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_Q6_K: k_dequant_q6k<<<(unsigned)((nblocks * 64 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        case GB_DT_Q8_0: k_dequant_q8_0<<<(unsigned)((nblocks * 32 + 255) / 256), 256, 0, st>>>(B, nblocks, out); break;
        default: return GB_EINVAL;
    }
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

extern "C" int gb_synth_blocks(int dtype, void* blocks, size_t nblocks, uint64_t seed, uint64_t stream_id,
                               void* stream) {
    if (!blocks) return GB_EINVAL;
    if (nblocks == 0) return GB_OK;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = (unsigned)((nblocks + 255) / 256);
    uint8_t* B = static_cast<uint8_t*>(blocks);
    switch (dtype) {
        case GB_DT_Q4_K:
            if (reinterpret_cast<uintptr_t>(blocks) & 15) return GB_EINVAL;
            k_synth_q4k<<<grid, 256, 0, st>>>(B, nblocks, seed, stream_id); break;
        case GB_DT_Q6_K:
            if (reinterpret_cast<uintptr_t>(blocks) & 1) return GB_EINVAL;
            k_synth_q6k<<<grid, 256, 0, st>>>(B, nblocks, seed, stream_id); break;
        case GB_DT_Q8_0:
            if (reinterpret_cast<uintptr_t>(blocks) & 1) return GB_EINVAL;
            k_synth_q8_0<<<grid, 256, 0, st>>>(B, nblocks, seed, stream_id); break;
        default: return GB_EINVAL;
    }
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
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
