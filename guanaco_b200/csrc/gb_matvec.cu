// gb_matvec.cu -- fused dequantise + matvec y = W x over GGUF Q4_K / Q6_K /
// Q8_0 blocks for batch-1 decode on sm_100a.
//
// Reference semantics: y[r] = sum_c dequant(W[r, c]) * x[c]
//   Q4_K  src/kernels/cpu/quant_matvec_q4_k.c:65-173 (w = d*sc*q - dmin*m)
//   Q6_K  src/kernels/cpu/quant_matvec_q6_k.c:43-98  (w = d*sc*(q - 32))
//   Q8_0  src/kernels/cpu/quant_matvec_q8_0.c:41-78  (w = d*q)
// The reference CUDA kernels these replace are matvec_q4k_kernel
// (src/kernels/cuda/matvec_q4k_cuda.cu:29-77) and matvec_q6k_kernel
// (src/kernels/cuda/cuda_layer_kernels.cu:26-75); there was no Q8_0 kernel.
//
// Design (B200):
//  * Memory: one producer warp per CTA streams row tiles from HBM into a
//    3-8 stage shared-memory ring with cp.async.bulk (one copy per row, one
//    row per producer lane, rows placed at a padded stride so 128-bit shared
//    reads are bank-conflict free), completion counted on mbarriers.  Bytes in flight per SM are set
//    by the ring depth (100-200 KB), not by registers.
//  * Math: on B200 the integer ALU, not HBM, limits a CUDA-core GEMV over
//    4-bit blocks (one mask per weight plus the fp32 FMA).  Q4_K and Q6_K
//    therefore run their multiply-accumulates on the int8 tensor cores:
//    mma.sync m16n8k32 u8 x s8 -> s32 with 16 weight rows per warp.  Weights
//    enter as exact u8 codes (one LOP3 per 4 Q4_K weights); x enters as three
//    int8 limbs x ~ s (x0 + x1 / 256 + x2 / 65536) with one scale s per
//    sub-block, which keeps fp32's 24 significant bits of every element; the
//    8 output columns of the first MMA of a k-step are 4 sub-blocks x 2
//    limbs, a second MMA on the same A fragment takes the third limb, so each
//    thread owns whole sub-blocks and applies their 6-bit / int8 block scales
//    in fp32.  The result matches an fp32 matvec to ~1e-6 relative.
//  * Q8_0 keeps a CUDA-core fp32 consumer (field extraction into exact
//    subnormal floats, FFMA2) on the same ring.
//  * Every mbarrier wait is bounded (2 s of %globaltimer); a timeout records
//    GB_ETIMEOUT in the device error word and the CTA winds down without
//    touching global memory it does not own.
#include "gb_common.cuh"
#include "gb_internal.h"
#include "gb_mt.cuh"
#include "gb_tc.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <map>
#include <mutex>

namespace gb {

constexpr int MV_CONSUMERS = 16;                      // consumer warps per CTA
constexpr int MV_THREADS = (MV_CONSUMERS + 1) * 32;   // + one producer warp
constexpr int MV_SMEM_MAX = 227 * 1024;
constexpr unsigned long long MV_WAIT_NS = 2000000000ull;

__device__ unsigned g_gb_device_err;

// ------------------------------------------------------------------ primitives
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sptr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* b, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sptr(b)), "r"(tx) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sptr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(sptr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of parity `parity`; false on timeout or when the CTA is
// already aborting (the caller then proceeds without the data).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (mbar_test(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        if (*abort_flag) return false;
        for (int i = 0; i < 32; i++)
            if (mbar_test(b, parity)) return true;
        if (gtimer() - t0 > MV_WAIT_NS) {
            *abort_flag = 1;
            atomicExch(&g_gb_device_err, (unsigned)(-GB_ETIMEOUT));
            return false;
        }
    }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(sptr(dst)), "l"(src), "r"(bytes), "r"(sptr(b))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync() {
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(MV_CONSUMERS * 32) : "memory");
}
// 8 bytes at a 2-byte-aligned shared address: two aligned words, one aligned
// half word, two funnel shifts (shift 0 or 16, so the read ends at p + 8).
struct Pair32 { uint32_t lo, hi; };
__device__ __forceinline__ Pair32 lds8_unaligned(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = *reinterpret_cast<const uint16_t*>(w + 2);
    return {__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh)};
}

// ------------------------------------------------------------------ geometry
// Work is cut into row groups of T rows (16 = one tensor-core tile); each
// group streams through the ring as nk sub-tiles of KC blocks.  Row r of a
// sub-tile sits at stage + r * RS + (segment_start & 15), RS = 16 (mod 128)
// for conflict-free 128-bit reads across the row groups of a warp.  CTA i
// processes groups i, i + grid, ...; accumulators live in registers across a
// group's sub-tiles.
struct MvGeom {
    int T;         // rows per group
    int KC;        // blocks per sub-tile
    int nk;        // sub-tiles per group
    int S;         // ring stages
    int RS;        // row stride inside a stage (bytes)
    int SB;        // bytes per stage
    int ngroups;
    int red_off, ring_off, bar_off;   // offsets inside dynamic shared memory
};

// Producer warp: per sub-tile, lane r issues the bulk copy of row r,
// [floor16(start), ceil16(end)) clamped to the matrix (the last < 16 bytes of
// a matrix whose size is not a multiple of 16 are copied by hand); lane 0
// first posts the stage's total transaction bytes on the full barrier.
__device__ void ring_producer(const uint8_t* __restrict__ W, int rows, int nb, size_t bbytes, const MvGeom& g,
                              uint8_t* ring, uint64_t* full, uint64_t* empty, volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    const size_t rb = (size_t)nb * bbytes;
    const size_t total = rb * (size_t)rows, tot16 = total & ~size_t(15);
    int it = 0;
    bool stop = false;
    for (int grp = blockIdx.x; grp < g.ngroups && !stop; grp += gridDim.x) {
        const int row0 = grp * g.T;
        const int nr = rows - row0 < g.T ? rows - row0 : g.T;
        for (int kc = 0; kc < g.nk; kc++, it++) {
            const int s = it % g.S, n = it / g.S;
            int ok = 1;
            if (n > 0 && lane == 0) ok = mbar_wait(&empty[s], (n - 1) & 1, abort_flag);
            if (!__shfl_sync(0xffffffffu, ok, 0)) { stop = true; break; }
            const int b0 = kc * g.KC, nblk = nb - b0 < g.KC ? nb - b0 : g.KC;
            uint8_t* stage = ring + (size_t)s * g.SB;
            size_t a = 0, e = 0;
            if (lane < nr) {
                const size_t start = (size_t)(row0 + lane) * rb + (size_t)b0 * bbytes, end = start + nblk * bbytes;
                a = start & ~size_t(15);
                e = (end + 15) & ~size_t(15);
                if (e > tot16) e = tot16;
                uint8_t* dst = stage + (size_t)lane * g.RS;
                for (size_t i = e > start ? e : start; i < end; i++) dst[i - a] = W[i];
                if (e < a) e = a;
            }
            uint32_t tx = (uint32_t)(e - a);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) tx += __shfl_xor_sync(0xffffffffu, tx, o);
            if (lane == 0) mbar_arrive_tx(&full[s], tx);
            __syncwarp();
            if (e > a) bulk_g2s(stage + (size_t)lane * g.RS, W + a, (uint32_t)(e - a), &full[s]);
        }
    }
    // every issued copy has landed before the producer warp leaves
    if (lane == 0)
        for (int j = it - g.S > 0 ? it - g.S : 0; j < it; j++) mbar_wait(&full[j % g.S], (j / g.S) & 1, abort_flag);
    __syncwarp();
}

// Offset of row r's data inside a sub-tile stage.
__device__ __forceinline__ size_t seg_lead(int row, int b0, size_t rb, size_t bbytes) {
    return ((size_t)row * rb + (size_t)b0 * bbytes) & 15;
}

// Per-CTA shared state layout, set up by kernel_prologue.
struct MvShared {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    int* cnt;
    volatile int* abort_flag;
    float* red;
};

__device__ __forceinline__ MvShared kernel_prologue(uint8_t* smem, const MvGeom& g) {
    MvShared sh;
    sh.red = reinterpret_cast<float*>(smem + g.red_off);
    sh.ring = smem + g.ring_off;
    sh.full = reinterpret_cast<uint64_t*>(smem + g.bar_off);
    sh.empty = sh.full + g.S;
    sh.cnt = reinterpret_cast<int*>(sh.empty + g.S);
    sh.abort_flag = sh.cnt + g.S + 2;
    if (threadIdx.x == 0) {
        for (int s = 0; s < g.S; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], MV_CONSUMERS);
        }
        for (int s = 0; s < g.S + 2; s++) sh.cnt[s] = 0;
        *sh.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    return sh;
}

// Group epilogue, run after the group's last stage was already released:
// red[slot][w][row] holds each consumer warp's row partials; the last warp to
// arrive sums the warps in order and writes y.  Slots rotate over S + 2
// groups: a warp cannot run more than S sub-tiles ahead of the slowest one
// (stage reuse waits for every warp), so a slot is never refilled while its
// finisher may still be reading it.
__device__ __forceinline__ void group_epilogue(const MvShared& sh, const MvGeom& g, int slot, int row0, int nrows,
                                               float* __restrict__ y, const float* __restrict__ residual) {
    const int lane = threadIdx.x & 31, WK = MV_CONSUMERS;
    float* rs = sh.red + (size_t)slot * WK * g.T;
    __syncwarp();            // every lane's partial-sum store precedes lane 0's ticket
    __threadfence_block();
    int last = 0;
    if (lane == 0) last = atomicAdd(&sh.cnt[slot], 1) == MV_CONSUMERS - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
        __threadfence_block();
        for (int r = lane; r < nrows; r += 32) {
            float v = 0.f;
#pragma unroll 4
            for (int k = 0; k < WK; k++) v += rs[k * g.T + r];
            y[row0 + r] = v + (residual ? residual[row0 + r] : 0.f);
        }
        __syncwarp();
        if (lane == 0) sh.cnt[slot] = 0;
    }
}

// ================================================================== Q4_K (MMA)
// Staged x per block b (256 columns), for mma u (0..3) x lohi (0..1):
//   xb[(b*8 + 2u + lohi)*8 + 2c + limb] = {limb of columns 64c + 32 lohi + 8u
//   + 0..3, + 4..7} -- the B-fragment pair of the lanes of column group c;
//   xs[b*8 + j]: x scale of sub-block j = 2c + lohi (the hi one divided by 16
//   because hi nibbles are masked in place as 16 q); xsum[b*8 + j]: sum of x
//   over sub-block j (for the dmin * m term).
// Lane (gq = lane >> 2, c = lane & 3) holds A rows gq and gq + 8 of its
// warp's 16-row group: k-slots 4c..4c+3 / 16+4c..16+4c+3 = the low (or high)
// nibbles of qs bytes 32c + 8u + 0..3 / 4..7, i.e. sub-block 2c (or 2c+1).
// The consumer warps split each sub-tile's blocks (warp w: blocks w, w+8, ..).
__global__ void __launch_bounds__(MV_THREADS)
k_mv_q4k(const uint8_t* __restrict__ W, int rows, int nb, const float* __restrict__ x, float* __restrict__ y,
         const float* __restrict__ residual, MvGeom g) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint2* xb = reinterpret_cast<uint2*>(smem);
    float* xs = reinterpret_cast<float*>(xb + (size_t)nb * 64);
    float* xsum = xs + (size_t)nb * 8;
    uint2* xb2 = reinterpret_cast<uint2*>(xsum + (size_t)nb * 8);   // third limb [(b*8 + 2u + lohi)*4 + c]
    const MvShared sh = kernel_prologue(smem, g);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == MV_CONSUMERS) {
        ring_producer(W, rows, nb, GB_Q4K_BYTES, g, sh.ring, sh.full, sh.empty, sh.abort_flag);
        return;
    }
    // ---- stage x: one warp per 32-column sub-block, one lane per column
    for (int e = warp; e < nb * 8; e += MV_CONSUMERS) {
        const int b = e >> 3, j = e & 7, cg = j >> 1, lohi = j & 1;
        const float v = x[b * 256 + 64 * cg + 32 * lohi + lane];
        const float mx = warp_max(fabsf(v));
        const float sum = warp_sum(v);
        int a0, a1, a2;
        limbs(v * (mx > 0.f ? 127.f / mx : 0.f), a0, a1, a2);
        uint8_t* dst = reinterpret_cast<uint8_t*>(xb + (size_t)((b * 8 + 2 * (lane >> 3) + lohi) * 8 + 2 * cg));
        dst[lane & 7] = (uint8_t)a0;
        dst[8 + (lane & 7)] = (uint8_t)a1;
        reinterpret_cast<uint8_t*>(xb2 + (size_t)((b * 8 + 2 * (lane >> 3) + lohi) * 4 + cg))[lane & 7] = (uint8_t)a2;
        if (lane == 0) {
            xs[e] = (mx / 127.f) * (lohi ? 0.0625f : 1.f);
            xsum[e] = sum;
        }
    }
    consumer_sync();

    const int gq = lane >> 2, c = lane & 3;
    const bool bact = c == (gq >> 1);   // this lane carries a nonzero B fragment
    const bool b2act = bact && !(gq & 1);   // ... and one of the third-limb MMA (column 2c)
    const int bsel = 2 * c + (gq & 1);
    const int sh8 = (c & 1) << 4;
    int it = 0, gi = 0;
    for (int grp = blockIdx.x; grp < g.ngroups; grp += gridDim.x) {
        const int row0 = grp * g.T;
        const int nrows = rows - row0 < g.T ? rows - row0 : g.T;
        const bool va = gq < nrows, vb = gq + 8 < nrows;
        float acc_a = 0.f, acc_b = 0.f;
        for (int kc = 0; kc < g.nk; kc++, it++) {
            const int s = it % g.S;
            mbar_wait(&sh.full[s], (it / g.S) & 1, sh.abort_flag);
            const int b0 = kc * g.KC, nblk = nb - b0 < g.KC ? nb - b0 : g.KC;
            const uint8_t* stage = sh.ring + (size_t)s * g.SB;
            const uint8_t* pa = stage + (size_t)(va ? gq : 0) * g.RS;        // Q4_K segments are 16-byte aligned
            const uint8_t* pb = stage + (size_t)(vb ? gq + 8 : 0) * g.RS;
            for (int bl = warp; bl < nblk; bl += MV_CONSUMERS) {
                const int b = b0 + bl;
                const uint8_t* ba = pa + (size_t)bl * GB_Q4K_BYTES;
                const uint8_t* bb = pb + (size_t)bl * GB_Q4K_BYTES;
                const uint4 ha = *reinterpret_cast<const uint4*>(ba);
                const uint4 hb = *reinterpret_cast<const uint4*>(bb);
                uint4 qa[2], qb[2];
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    qa[v] = va ? *reinterpret_cast<const uint4*>(ba + 16 + 32 * c + 16 * v) : make_uint4(0, 0, 0, 0);
                    qb[v] = vb ? *reinterpret_cast<const uint4*>(bb + 16 + 32 * c + 16 * v) : make_uint4(0, 0, 0, 0);
                }
                int4 cl[2] = {make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0)};
                int4 ch[2] = {make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0)};
                int4 cl3 = make_int4(0, 0, 0, 0), ch3 = make_int4(0, 0, 0, 0);
                const uint2* xbb = xb + (size_t)b * 64;
                const uint2* xbb2 = xb2 + (size_t)b * 32;
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const uint32_t wa0 = (u & 1) ? qa[u >> 1].z : qa[u >> 1].x;
                    const uint32_t wa1 = (u & 1) ? qa[u >> 1].w : qa[u >> 1].y;
                    const uint32_t wb0 = (u & 1) ? qb[u >> 1].z : qb[u >> 1].x;
                    const uint32_t wb1 = (u & 1) ? qb[u >> 1].w : qb[u >> 1].y;
                    uint2 blo = make_uint2(0, 0), bhi = make_uint2(0, 0), tlo = make_uint2(0, 0), thi = make_uint2(0, 0);
                    if (bact) {
                        blo = xbb[(2 * u) * 8 + bsel];
                        bhi = xbb[(2 * u + 1) * 8 + bsel];
                    }
                    if (b2act) {
                        tlo = xbb2[(2 * u) * 4 + c];
                        thi = xbb2[(2 * u + 1) * 4 + c];
                    }
                    mma_u8s8(cl[u & 1], wa0 & 0x0F0F0F0Fu, wb0 & 0x0F0F0F0Fu, wa1 & 0x0F0F0F0Fu, wb1 & 0x0F0F0F0Fu,
                             blo.x, blo.y);
                    mma_u8s8(ch[u & 1], wa0 & 0xF0F0F0F0u, wb0 & 0xF0F0F0F0u, wa1 & 0xF0F0F0F0u, wb1 & 0xF0F0F0F0u,
                             bhi.x, bhi.y);
                    mma_u8s8(cl3, wa0 & 0x0F0F0F0Fu, wb0 & 0x0F0F0F0Fu, wa1 & 0x0F0F0F0Fu, wb1 & 0x0F0F0F0Fu, tlo.x, tlo.y);
                    mma_u8s8(ch3, wa0 & 0xF0F0F0F0u, wb0 & 0xF0F0F0F0u, wa1 & 0xF0F0F0F0u, wb1 & 0xF0F0F0F0u, thi.x, thi.y);
                }
                const int4 clo = make_int4(cl[0].x + cl[1].x, cl[0].y + cl[1].y, cl[0].z + cl[1].z, cl[0].w + cl[1].w);
                const int4 chi = make_int4(ch[0].x + ch[1].x, ch[0].y + ch[1].y, ch[0].z + ch[1].z, ch[0].w + ch[1].w);
                // sub-blocks 2c (lo) and 2c+1 (hi): scales and mins of rows a and b
                const float2 sxs = *reinterpret_cast<const float2*>(xs + b * 8 + 2 * c);
                const float2 sxm = *reinterpret_cast<const float2*>(xsum + b * 8 + 2 * c);
#pragma unroll
                for (int w = 0; w < 2; w++) {
                    const uint4 h = w ? hb : ha;
                    const uint32_t scw = c < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
                    const uint32_t mw = c < 2 ? (h.z & 0x3F3F3F3Fu)
                                              : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
                    const float sc_lo = (float)((scw >> sh8) & 0xFFu), sc_hi = (float)((scw >> (sh8 + 8)) & 0xFFu);
                    const float m_lo = (float)((mw >> sh8) & 0xFFu), m_hi = (float)((mw >> (sh8 + 8)) & 0xFFu);
                    const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                    const int c0 = w ? clo.z : clo.x, c1 = w ? clo.w : clo.y;
                    const int e0 = w ? chi.z : chi.x, e1 = w ? chi.w : chi.y;
                    const int c2 = w ? cl3.z : cl3.x, e2 = w ? ch3.z : ch3.x;
                    const float dlo = fmaf((float)c2, 1.0f / 65536.0f, fmaf((float)c1, 0.00390625f, (float)c0));
                    const float dhi = fmaf((float)e2, 1.0f / 65536.0f, fmaf((float)e1, 0.00390625f, (float)e0));
                    const float part = dm.x * (sc_lo * sxs.x * dlo + sc_hi * sxs.y * dhi) -
                                       dm.y * (m_lo * sxm.x + m_hi * sxm.y);
                    if (w) acc_b += part; else acc_a += part;
                }
            }
            __syncwarp();   // release the stage as soon as this warp is done with it
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        // reduce over the 4 column-group lanes of each row, then across warps
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 2);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 2);
        const int slot = gi++ % (g.S + 2);
        float* rs = sh.red + (size_t)slot * MV_CONSUMERS * g.T + warp * g.T;
        if (c == 0) {
            if (va) rs[gq] = acc_a;
            if (vb) rs[gq + 8] = acc_b;
        }
        group_epilogue(sh, g, slot, row0, nrows, y, residual);
    }
}

// ================================================================== Q6_K (MMA)
// mma (n, G) of a block: half n (0..1), group G (0..3); the lanes of column
// group c hold weights l in [8c, 8c+8) of group G (columns 128n + 32G + l),
// q = (ql nibble | qh bits << 4), a u8 code 0..63; their sub-block is
// 8n + 2G + (c >> 1) (16 weights, int8 scale).
// Staged x per block: xb[(b*8 + 4n + G)*8 + 2c + limb] (B-fragment pair of
// columns 128n + 32G + 8c + 0..3, 4..7), xs[b*16 + 8n + 2G + (c>>1)] = x
// scale of the 16-column sub-block, xs32[b*32 + (4n + G)*4 + c] = 32 * sum of
// the quantised x over the lanes' 8 columns (the -32 offset of the codes).
__global__ void __launch_bounds__(MV_THREADS)
k_mv_q6k(const uint8_t* __restrict__ W, int rows, int nb, const float* __restrict__ x, float* __restrict__ y,
         const float* __restrict__ residual, MvGeom g) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint2* xb = reinterpret_cast<uint2*>(smem);
    float* xs = reinterpret_cast<float*>(xb + (size_t)nb * 64);
    float* xs32 = xs + (size_t)nb * 16;
    uint2* xb2 = reinterpret_cast<uint2*>(xs32 + (size_t)nb * 32);   // third limb [(b*8 + 4n + G)*4 + c]
    const MvShared sh = kernel_prologue(smem, g);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t rb = (size_t)nb * GB_Q6K_BYTES;
    if (warp == MV_CONSUMERS) {
        ring_producer(W, rows, nb, GB_Q6K_BYTES, g, sh.ring, sh.full, sh.empty, sh.abort_flag);
        return;
    }
    // ---- stage x: one warp per 32 columns (b, n, G) = two 16-column
    // sub-blocks, one lane per column; column group c = lane >> 3
    for (int e = warp; e < nb * 8; e += MV_CONSUMERS) {
        const int b = e >> 3, n = (e >> 2) & 1, G = e & 3;
        const float v = x[b * 256 + 128 * n + 32 * G + lane];
        float mx = fabsf(v);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int a0, a1, a2;
        limbs(v * (mx > 0.f ? 127.f / mx : 0.f), a0, a1, a2);
        // 8-column sums of the quantised values: the -32 code offset then
        // applies to the same x the codes multiply (see mt_quantise4)
        float s8 = limb_value(a0, a1, a2);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) s8 += __shfl_xor_sync(0xffffffffu, s8, o);
        s8 *= mx / 127.f;
        const int c = lane >> 3;
        uint8_t* dst = reinterpret_cast<uint8_t*>(xb + (size_t)((b * 8 + 4 * n + G) * 8 + 2 * c));
        dst[lane & 7] = (uint8_t)a0;
        dst[8 + (lane & 7)] = (uint8_t)a1;
        reinterpret_cast<uint8_t*>(xb2 + (size_t)((b * 8 + 4 * n + G) * 4 + c))[lane & 7] = (uint8_t)a2;
        if ((lane & 15) == 0) xs[b * 16 + 8 * n + 2 * G + (lane >> 4)] = mx / 127.f;
        if ((lane & 7) == 0) xs32[b * 32 + (4 * n + G) * 4 + c] = 32.f * s8;
    }
    consumer_sync();

    const int gq = lane >> 2, c = lane & 3;
    const bool bact = c == (gq >> 1);
    const bool b2act = bact && !(gq & 1);
    const int bsel = 2 * c + (gq & 1);
    int it = 0, gi = 0;
    for (int grp = blockIdx.x; grp < g.ngroups; grp += gridDim.x) {
        const int row0 = grp * g.T;
        const int nrows = rows - row0 < g.T ? rows - row0 : g.T;
        const bool va = gq < nrows, vb = gq + 8 < nrows;
        const int ia = va ? gq : 0, ib = vb ? gq + 8 : 0;
        float acc_a = 0.f, acc_b = 0.f;
        for (int kc = 0; kc < g.nk; kc++, it++) {
            const int s = it % g.S;
            mbar_wait(&sh.full[s], (it / g.S) & 1, sh.abort_flag);
            const int b0 = kc * g.KC, nblk = nb - b0 < g.KC ? nb - b0 : g.KC;
            const uint8_t* stage = sh.ring + (size_t)s * g.SB;
            const uint8_t* pa = stage + (size_t)ia * g.RS + seg_lead(row0 + ia, b0, rb, GB_Q6K_BYTES);
            const uint8_t* pb = stage + (size_t)ib * g.RS + seg_lead(row0 + ib, b0, rb, GB_Q6K_BYTES);
            for (int bl = warp; bl < nblk; bl += MV_CONSUMERS) {
                const int b = b0 + bl;
                const uint8_t* ba = pa + (size_t)bl * GB_Q6K_BYTES;
                const uint8_t* bb = pb + (size_t)bl * GB_Q6K_BYTES;
                const float da = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(ba + 208)));
                const float db = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(bb + 208)));
                const uint2* xbb = xb + (size_t)b * 64;
                const uint2* xbb2 = xb2 + (size_t)b * 32;
#pragma unroll
                for (int n = 0; n < 2; n++) {
                    Pair32 qa0 = {0, 0}, qa1 = {0, 0}, ha = {0, 0}, qb0 = {0, 0}, qb1 = {0, 0}, hb = {0, 0};
                    if (va) {
                        qa0 = lds8_unaligned(ba + 64 * n + 8 * c);
                        qa1 = lds8_unaligned(ba + 64 * n + 32 + 8 * c);
                        ha = lds8_unaligned(ba + 128 + 32 * n + 8 * c);
                    }
                    if (vb) {
                        qb0 = lds8_unaligned(bb + 64 * n + 8 * c);
                        qb1 = lds8_unaligned(bb + 64 * n + 32 + 8 * c);
                        hb = lds8_unaligned(bb + 128 + 32 * n + 8 * c);
                    }
#pragma unroll
                    for (int G = 0; G < 4; G++) {
                        // a0: row a word 0, a1: row b word 0, a2: row a word 1, a3: row b word 1
                        uint32_t A[4];
#pragma unroll
                        for (int t = 0; t < 4; t++) {
                            const Pair32& ql = (t & 1) ? ((G & 1) ? qb1 : qb0) : ((G & 1) ? qa1 : qa0);
                            const Pair32& qh = (t & 1) ? hb : ha;
                            const uint32_t lw = (t >> 1) ? ql.hi : ql.lo;
                            const uint32_t hw = (t >> 1) ? qh.hi : qh.lo;
                            const uint32_t nib = (G >> 1) ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
                            const uint32_t hi2 = G == 0 ? (hw << 4) : G == 1 ? (hw << 2) : G == 2 ? hw : (hw >> 2);
                            A[t] = nib | (hi2 & 0x30303030u);
                        }
                        uint2 bf = make_uint2(0, 0), bf2 = make_uint2(0, 0);
                        if (bact) bf = xbb[(4 * n + G) * 8 + bsel];
                        if (b2act) bf2 = xbb2[(4 * n + G) * 4 + c];
                        int4 cc = make_int4(0, 0, 0, 0), cc2 = make_int4(0, 0, 0, 0);
                        mma_u8s8(cc, A[0], A[1], A[2], A[3], bf.x, bf.y);
                        mma_u8s8(cc2, A[0], A[1], A[2], A[3], bf2.x, bf2.y);
                        const int sb = 8 * n + 2 * G + (c >> 1);
                        const float xsc = xs[b * 16 + sb];
                        const float x32 = xs32[b * 32 + (4 * n + G) * 4 + c];
                        const float sca = (float)(int)(int8_t)ba[192 + sb];
                        const float scb = (float)(int)(int8_t)bb[192 + sb];
                        const float dla = fmaf((float)cc2.x, 1.0f / 65536.0f, fmaf((float)cc.y, 0.00390625f, (float)cc.x));
                        const float dlb = fmaf((float)cc2.z, 1.0f / 65536.0f, fmaf((float)cc.w, 0.00390625f, (float)cc.z));
                        acc_a = fmaf(da * sca, fmaf(xsc, dla, -x32), acc_a);
                        acc_b = fmaf(db * scb, fmaf(xsc, dlb, -x32), acc_b);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 2);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 2);
        const int slot = gi++ % (g.S + 2);
        float* rs = sh.red + (size_t)slot * MV_CONSUMERS * g.T + warp * g.T;
        if (c == 0) {
            if (va) rs[gq] = acc_a;
            if (vb) rs[gq + 8] = acc_b;
        }
        group_epilogue(sh, g, slot, row0, nrows, y, residual);
    }
}

// ================================================================== Q8_0 (CUDA cores)
// Lane map per warp chunk of 8 blocks: block = lane>>2, s = lane&3 -> quants
// [8s, 8s+8).  Quants are read as unsigned bytes u = q + 128 (XOR 0x80) and
// masked in place into exact subnormal floats u * 2^(p-149); x carries the
// compensating power of two so products land at u * x * 2^-49.  Each warp
// owns whole rows of the 16-row group (row w, w + 16/..), so the cross-warp
// reduction only moves finished sums.
constexpr float P100 = 0x1p100f, P92 = 0x1p92f, P84 = 0x1p84f, P49 = 0x1p49f;

__global__ void __launch_bounds__(MV_THREADS)
k_mv_q8_0(const uint8_t* __restrict__ W, int rows, int nb, const float* __restrict__ x, float* __restrict__ y,
          const float* __restrict__ residual, MvGeom g) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nchunks = (nb + 7) / 8;
    float4* xs = reinterpret_cast<float4*>(smem);      // [chunk][lane][2] prescaled x
    float* sx = reinterpret_cast<float*>(xs + (size_t)nchunks * 64);   // [chunk][lane] 128 * sum x
    const MvShared sh = kernel_prologue(smem, g);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t rb = (size_t)nb * GB_Q80_BYTES;
    if (warp == MV_CONSUMERS) {
        ring_producer(W, rows, nb, GB_Q80_BYTES, g, sh.ring, sh.full, sh.empty, sh.abort_flag);
        return;
    }
    for (int e = tid; e < nchunks * 32; e += MV_CONSUMERS * 32) {
        const int c = e >> 5, L = e & 31, b = c * 8 + (L >> 2);
        float4 u = make_float4(0.f, 0.f, 0.f, 0.f), v = u;
        if (b < nb) {
            const float4* p = reinterpret_cast<const float4*>(x + b * 32 + 8 * (L & 3));
            u = p[0];
            v = p[1];
        }
        const int sw = (L >> 2) & 1;
        xs[(size_t)e * 2 + (0 ^ sw)] = make_float4(u.x * P100, u.y * P92, u.z * P84, u.w * P84);
        xs[(size_t)e * 2 + (1 ^ sw)] = make_float4(v.x * P100, v.y * P92, v.z * P84, v.w * P84);
        sx[e] = 128.f * (((u.x + u.y) + (u.z + u.w)) + ((v.x + v.y) + (v.z + v.w)));
    }
    consumer_sync();

    const int sw = (lane >> 2) & 1;
    int it = 0, gi = 0;
    for (int grp = blockIdx.x; grp < g.ngroups; grp += gridDim.x) {
        const int row0 = grp * g.T;
        const int nrows = rows - row0 < g.T ? rows - row0 : g.T;
        float acc[2] = {0.f, 0.f};
        for (int kc = 0; kc < g.nk; kc++, it++) {
            const int s = it % g.S;
            mbar_wait(&sh.full[s], (it / g.S) & 1, sh.abort_flag);
            const int b0 = kc * g.KC, nblk = nb - b0 < g.KC ? nb - b0 : g.KC;
            const uint8_t* stage = sh.ring + (size_t)s * g.SB;
#pragma unroll
            for (int rr = 0; rr < 16 / MV_CONSUMERS; rr++) {
                const int lr = warp + MV_CONSUMERS * rr;
                if (lr >= nrows) continue;
                const uint8_t* prow = stage + (size_t)lr * g.RS + seg_lead(row0 + lr, b0, rb, GB_Q80_BYTES);
                for (int cl = 0; cl * 8 < nblk; cl++) {
                    const int bl = cl * 8 + (lane >> 2);
                    if (bl >= nblk) continue;
                    const int c = (b0 + bl) >> 3;   // global chunk (KC is a multiple of 8)
                    const uint8_t* blk = prow + (size_t)bl * GB_Q80_BYTES;
                    const Pair32 q = lds8_unaligned(blk + 2 + 8 * (lane & 3));
                    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
                    const float4 x0 = xs[((size_t)c * 32 + lane) * 2 + (0 ^ sw)];
                    const float4 x1 = xs[((size_t)c * 32 + lane) * 2 + (1 ^ sw)];
                    float2 a = make_float2(0.f, 0.f);
                    const uint32_t u0 = q.lo ^ 0x80808080u, u1 = q.hi ^ 0x80808080u;
                    a = __ffma2_rn(make_float2(__uint_as_float(u0 & 0xFFu), __uint_as_float(u0 & 0xFF00u)), make_float2(x0.x, x0.y), a);
                    a = __ffma2_rn(make_float2(__uint_as_float(u0 & 0xFF0000u), __uint_as_float(__byte_perm(u0, 0u, 0x4344u))), make_float2(x0.z, x0.w), a);
                    a = __ffma2_rn(make_float2(__uint_as_float(u1 & 0xFFu), __uint_as_float(u1 & 0xFF00u)), make_float2(x1.x, x1.y), a);
                    a = __ffma2_rn(make_float2(__uint_as_float(u1 & 0xFF0000u), __uint_as_float(__byte_perm(u1, 0u, 0x4344u))), make_float2(x1.z, x1.w), a);
                    acc[rr] += d * fmaf(a.x + a.y, P49, -sx[c * 32 + lane]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        const int slot = gi++ % (g.S + 2);
        // whole rows per warp: the owner fills every warp slot of its rows
        // (its sum in slot 0, zeros elsewhere) so the shared epilogue applies
#pragma unroll
        for (int rr = 0; rr < 16 / MV_CONSUMERS; rr++) {
            const float v = warp_sum(acc[rr]);
            const int lr = warp + MV_CONSUMERS * rr;
            if (lane == 0) {
                for (int k = 0; k < MV_CONSUMERS; k++)
                    if (lr < nrows) sh.red[(size_t)slot * MV_CONSUMERS * g.T + k * g.T + lr] = k == 0 ? v : 0.f;
            }
        }
        group_epilogue(sh, g, slot, row0, nrows, y, residual);
    }
}

// ================================================================== Q5_K / F16 (CUDA cores)
// Formats the reference does not compute (its loader rejects them): GGML's
// Q5_K (block of 256: d, dmin, 12 packed 6-bit scales / mins as Q4_K, qh[32]
// fifth bits, qs[128] low nibbles; w = d sc q - dmin m, q = nibble + 16 x bit
// j of qh for sub-block j) and plain fp16 rows.  x is staged in shared memory
// as fp32 (Q5_K also with per-8-column sums); each consumer warp owns one row
// of the 16-row group.  Q5_K: lane (j = lane / 4, c = lane % 4) takes columns
// 32 j + 8 c .. + 7 of every block, sum = d sc (q . x) - dmin m (sum x).  F16:
// lane l takes 8 consecutive halves of every 256-column chunk.
template <int DT>
__global__ void __launch_bounds__(MV_THREADS)
k_mv_plain(const uint8_t* __restrict__ W, int rows, int nb, const float* __restrict__ x, float* __restrict__ y,
           const float* __restrict__ residual, MvGeom g) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr bool Q5 = DT == GB_DT_Q5_K;
    constexpr int WIDTH = Q5 ? 256 : 32, BYTES = Q5 ? GB_Q5K_BYTES : GB_F16_BYTES;
    const int K = nb * WIDTH;
    float* xs = reinterpret_cast<float*>(smem);   // [K] fp32, then (Q5_K) [K / 8] sums
    float* x8 = xs + K;
    const MvShared sh = kernel_prologue(smem, g);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t rb = (size_t)nb * BYTES;
    if (warp == MV_CONSUMERS) {
        ring_producer(W, rows, nb, BYTES, g, sh.ring, sh.full, sh.empty, sh.abort_flag);
        return;
    }
    for (int e = tid; e < K / 4; e += MV_CONSUMERS * 32) {
        const float4 v = reinterpret_cast<const float4*>(x)[e];
        reinterpret_cast<float4*>(xs)[e] = v;
        if (Q5) {   // sums of 8 columns: two float4 per sum, added by the even thread
            const float h = (v.x + v.y) + (v.z + v.w);
            const float o = __shfl_down_sync(0xffffffffu, h, 1);
            if ((e & 1) == 0) x8[e >> 1] = h + o;
        }
    }
    consumer_sync();
    int it = 0, gi = 0;
    const int lr = warp;   // 16-row groups, one row per consumer warp
    for (int grp = blockIdx.x; grp < g.ngroups; grp += gridDim.x) {
        const int row0 = grp * g.T;
        const int nrows = rows - row0 < g.T ? rows - row0 : g.T;
        float acc = 0.f;
        for (int kc = 0; kc < g.nk; kc++, it++) {
            const int s = it % g.S;
            mbar_wait(&sh.full[s], (it / g.S) & 1, sh.abort_flag);
            const int b0 = kc * g.KC, nblk = nb - b0 < g.KC ? nb - b0 : g.KC;
            if (lr < nrows) {
                // rows of 176 / 64-byte blocks start 16-byte aligned in the stage
                const uint8_t* prow = sh.ring + (size_t)s * g.SB + (size_t)lr * g.RS + seg_lead(row0 + lr, b0, rb, BYTES);
                if constexpr (Q5) {
                    const int j = lane >> 2, c8 = 8 * (lane & 3);
                    for (int bl = 0; bl < nblk; bl++) {
                        const uint8_t* blk = prow + (size_t)bl * BYTES;
                        const uint4 hd = *reinterpret_cast<const uint4*>(blk);
                        const uint2 qh = *reinterpret_cast<const uint2*>(blk + 16 + c8);
                        const uint2 qs = *reinterpret_cast<const uint2*>(blk + 48 + 32 * (j >> 1) + c8);
                        const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
                        auto sbyte = [&](int i) {
                            const uint32_t w = i < 4 ? hd.y : (i < 8 ? hd.z : hd.w);
                            return (w >> (8 * (i & 3))) & 0xFFu;
                        };
                        uint32_t sc, mn;
                        if (j < 4) { sc = sbyte(j) & 63; mn = sbyte(j + 4) & 63; }
                        else { sc = (sbyte(j + 4) & 0xF) | ((sbyte(j - 4) >> 6) << 4); mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4); }
                        const int col = (b0 + bl) * 256 + 32 * j + c8;
                        const float4 xa = *reinterpret_cast<const float4*>(xs + col);
                        const float4 xb = *reinterpret_cast<const float4*>(xs + col + 4);
                        const uint32_t q0 = ((qs.x >> (4 * (j & 1))) & 0x0F0F0F0Fu) | (((qh.x >> j) & 0x01010101u) << 4);
                        const uint32_t q1 = ((qs.y >> (4 * (j & 1))) & 0x0F0F0F0Fu) | (((qh.y >> j) & 0x01010101u) << 4);
                        float dot = tc::byte_as_float<0>(q0, 0.f) * xa.x;
                        dot = fmaf(tc::byte_as_float<1>(q0, 0.f), xa.y, dot);
                        dot = fmaf(tc::byte_as_float<2>(q0, 0.f), xa.z, dot);
                        dot = fmaf(tc::byte_as_float<3>(q0, 0.f), xa.w, dot);
                        dot = fmaf(tc::byte_as_float<0>(q1, 0.f), xb.x, dot);
                        dot = fmaf(tc::byte_as_float<1>(q1, 0.f), xb.y, dot);
                        dot = fmaf(tc::byte_as_float<2>(q1, 0.f), xb.z, dot);
                        dot = fmaf(tc::byte_as_float<3>(q1, 0.f), xb.w, dot);
                        acc = fmaf(d * (float)sc, dot, acc);
                        acc = fmaf(-(dmin * (float)mn), x8[col >> 3], acc);
                    }
                } else {
                    for (int c = 0; c * 8 < nblk; c++) {
                        if (c * 8 + (lane >> 2) >= nblk) continue;
                        const uint4 h = *reinterpret_cast<const uint4*>(prow + (size_t)c * 512 + 16 * lane);
                        const int col = (b0 + 8 * c) * 32 + 8 * lane;
                        const float4 xa = *reinterpret_cast<const float4*>(xs + col);
                        const float4 xb = *reinterpret_cast<const float4*>(xs + col + 4);
                        const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                        const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                        const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&h.z));
                        const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&h.w));
                        acc = fmaf(w0.x, xa.x, acc);
                        acc = fmaf(w0.y, xa.y, acc);
                        acc = fmaf(w1.x, xa.z, acc);
                        acc = fmaf(w1.y, xa.w, acc);
                        acc = fmaf(w2.x, xb.x, acc);
                        acc = fmaf(w2.y, xb.y, acc);
                        acc = fmaf(w3.x, xb.z, acc);
                        acc = fmaf(w3.y, xb.w, acc);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
        }
        const int slot = gi++ % (g.S + 2);
        const float v = warp_sum(acc);
        if (lane == 0 && lr < nrows)   // whole rows per warp: the owner's sum in slot 0, zeros elsewhere
            for (int k = 0; k < MV_CONSUMERS; k++)
                sh.red[(size_t)slot * MV_CONSUMERS * g.T + k * g.T + lr] = k == 0 ? v : 0.f;
        group_epilogue(sh, g, slot, row0, nrows, y, residual);
    }
}

// Up to MT_MAXM matrices of one format and one column count that share x run
// as one launch: their (group, item) sequences are concatenated, matrix m
// owning the global 32-row groups [gbase[m], gbase[m + 1]).
constexpr int MT_MAXM = 3;
struct MtArgs {
    const float* x;
    float* y[MT_MAXM];
    const float* residual[MT_MAXM];
    int rows[MT_MAXM];
    int gbase[MT_MAXM + 1];
    int nm;
    float* part;        // [ncta][2][MT_GR] stream-K partial rows
    unsigned* tickets;  // [total groups], zero between launches
    int nb, T, ncta, S;
    int ibase[MT_MAXM + 1];   // first item of matrix m (T = ibase[nm])
    int nchm[MT_MAXM];        // items per 32-row group of matrix m
    int fmt[MT_MAXM];         // matrix m is Q6_K (mixed-format launches)
    int unit;           // split granularity in items: 1, or the items per group (whole groups, no workspace)
    // x transform applied while quantising (MV_X_*): RMSNorm with weight nw
    // and eps, or silu(x) * x2
    int xmode;
    const float* nw;
    const float* x2;
    float eps;
    MvTp tp;            // tensor-parallel exchange (push_call / in_call < 0: none)
    const uint8_t* xpre;   // MV_X_PREQ: x already quantised
    // gate / up: items interleaved (2 g = gate group g, 2 g + 1 = up group g),
    // silu(gate) * up quantised into swq_out (swq_K columns); swq_tk: one
    // ticket per group for pairs whose halves end in different CTAs
    uint8_t* swq_out;
    unsigned* swq_tk;
    int swq_K;
    // c1 > 0: CTAs [0, c1) take one whole group of n1 items each (the
    // leading matrices), the other CTAs split the rest (one item per group)
    int c1, n1;
    int l2pf;           // boxes past the ring prefetched into L2 at the start
};

// y row of matrix m: to y, or (tensor-parallel push) as {value, epoch} to
// slot [rank] of every rank's receive buffer
__device__ __forceinline__ void mt_put(const MtArgs& a, int m, int row, float v, unsigned ep) {
    if (a.tp.push_call >= 0) {
        const size_t off = ((size_t)(ep & 1) * a.tp.world + a.tp.rank) * a.tp.H + row;
        for (int q = 0; q < a.tp.world; q++) ll_store(static_cast<uint2*>(a.tp.peers[q]) + off, v, ep);
    } else {
        a.y[m][row] = v;
    }
}

// A launch whose matrices mix Q4_K and Q6_K (e.g. q, k and v): stage slots
// sized for the larger stage, each stage consumed by its matrix's format.
struct MtMix {
    static constexpr int NC = 16;
    static_assert(MtQ4K::NC == NC && MtQ6K::NC == NC, "one consumer layout");
    static constexpr int STG = MtQ4K::STG > MtQ6K::STG ? MtQ4K::STG : MtQ6K::STG;
    static constexpr bool S16 = true;
};
static_assert(MtQ4K::SI == 1 && MtQ6K::SI == 1, "one split item per stage");

// matrix, group within it and item within the group of item t
__device__ __forceinline__ void mt_locate(const MtArgs& a, int t, int& m, int& g, int& it) {
    if (a.swq_out) {   // gate / up pairs interleaved, one item per group
        m = t & 1;
        g = t >> 1;
        it = 0;
        return;
    }
    m = t >= a.ibase[1] ? (t >= a.ibase[2] ? 2 : 1) : 0;
    const int u = t - a.ibase[m];
    g = u / a.nchm[m];
    it = u - g * a.nchm[m];
}

template <class F>
__global__ void __launch_bounds__((F::NC + 1) * 32, 1) k_mvt(const __grid_constant__ CUtensorMap tm0,
                                                            const __grid_constant__ CUtensorMap tm1,
                                                            const __grid_constant__ CUtensorMap tm2, const MtArgs a) {
    constexpr int MT_NC = F::NC;
    constexpr bool MIXED = std::is_same<F, MtMix>::value;
    constexpr bool FQ6 = std::is_same<F, MtQ6K>::value;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.nb, K = nb * 256, S = a.S;
    const int NSLOT = S + 2;
    // shared layout: ring [S][F::STG] | x | zero[64] | red [NSLOT][MT_NC][MT_GR] | cnt | barriers
    const uint32_t sbase = sptr(smem);
    const uint32_t xq_off = (uint32_t)S * F::STG;
    const uint32_t xq_bytes = (uint32_t)mt_xq_bytes(K, F::S16);
    const uint32_t zero_off = xq_off + ((xq_bytes + 15) & ~15u);
    float* red = reinterpret_cast<float*>(smem + zero_off + MT_ZERO);
    unsigned* cnt = reinterpret_cast<unsigned*>(red + NSLOT * MT_NC * MT_GR);
    const uint32_t bar_full = (sptr(cnt + NSLOT) + 15) & ~7u;
    const uint32_t bar_empty = bar_full + 8 * S;
    // gate values of the CTA's last two pairs, for the SwiGLU quantisation
    float* stash = reinterpret_cast<float*>(smem + ((bar_empty + 8 * S - sbase + 15) & ~15u));
    const int c0 = blockIdx.x;
    const int TU = a.T / a.unit;
    auto range_start = [&](int c) {
        if (a.c1)
            return c <= a.c1 ? c * a.n1 : a.c1 * a.n1 + mt_start(c - a.c1, a.T - a.c1 * a.n1, a.ncta - a.c1);
        return mt_start(c, TU, a.ncta) * a.unit;
    };
    const int t0 = range_start(c0), t1 = range_start(c0 + 1);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbs_init(bar_full + 8 * s, 1);
            mbs_init(bar_empty + 8 * s, MT_NC);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < NSLOT; i += blockDim.x) cnt[i] = 0;
    if (threadIdx.x < MT_ZERO / 4) reinterpret_cast<uint32_t*>(smem + zero_off)[threadIdx.x] = 0;
    __syncthreads();
    griddep_launch();

    if (warp == MT_NC) {   // ---- producer: one elected lane streams the stage boxes
        if (lane == 0) {
            bool ok = true;
            int i = 0;
            for (int t = t0; t < t1; i++, t++) {   // one item (one box) per stage
                int m, g, it;
                mt_locate(a, t, m, g, it);
                const int s = i % S;
                if (i >= S && !(ok = mbs_wait(bar_empty + 8 * s, ((i / S) - 1) & 1, &g_gb_device_err))) break;
                const CUtensorMap* tm = m == 0 ? &tm0 : (m == 1 ? &tm1 : &tm2);
                const bool q6 = MIXED ? a.fmt[m] != 0 : FQ6;
                // z: 16-block units of blocks (Q4_K), 8-block runs (Q6_K)
                mbs_expect(bar_full + 8 * s, q6 ? MtQ6K::ITEM : MtQ4K::ITEM);
                tma_load_3d(sbase + s * F::STG, tm, 0, g * MT_GR, q6 ? it : it * MtQ4K::IG, bar_full + 8 * s);
                if (i == S - 1 && a.l2pf > 0) {
                    // the ring is full and the consumers are still waiting
                    // for x: pull this CTA's next boxes into L2 so HBM keeps
                    // streaming through the wait
                    for (int k = 1; k <= a.l2pf && t + k < t1; k++) {
                        int m2, g2, it2;
                        mt_locate(a, t + k, m2, g2, it2);
                        const CUtensorMap* tm2p = m2 == 0 ? &tm0 : (m2 == 1 ? &tm1 : &tm2);
                        const bool q62 = MIXED ? a.fmt[m2] != 0 : FQ6;
                        tma_prefetch_3d(tm2p, 0, g2 * MT_GR, q62 ? it2 : it2 * MtQ4K::IG);
                    }
                }
            }
            // do not retire while a box is still landing in this CTA's ring
            for (int k = i > S ? i - S : 0; ok && k < i; k++) ok = mbs_wait(bar_empty + 8 * (k % S), (k / S) & 1, &g_gb_device_err);
        }
        return;
    }

    // ---- consumers
    // the RMSNorm weight does not depend on the previous kernel: read it
    // before the wait (the one-pass quantiser keeps it in registers)
    const bool rms1 = a.xmode == MV_X_RMSNORM && K / 4 <= MT_XU * MT_NC * 32;
    float4 nwr[MT_XU];
    if (rms1) mt_load_norm_w<MT_NC>(a, K, threadIdx.x, nwr);
    griddep_wait();
    uint8_t* xq = smem + xq_off;
    // epochs of the tensor-parallel exchanges (the step counter is written
    // by the step's first kernel, complete by now)
    unsigned ep_push = 0, ep_in = 0;
    if (a.tp.push_call >= 0 || a.tp.in_call >= 0) {
        const unsigned long long sc = *a.tp.step * (unsigned long long)a.tp.calls;
        ep_push = (unsigned)(sc + a.tp.push_call + 1);
        ep_in = (unsigned)(sc + a.tp.in_call + 1);
    }
    // RMSNorm: one pass over x and the weight when every thread can hold its
    // share in registers (K <= 8192), else a scale pass and a quantise pass
    if (a.xmode == MV_X_PREQ) {   // quantised by the producing matvec: copy it in
        const int n16 = mt_xq_bytes(K, F::S16) / 16;
        const uint4* src = reinterpret_cast<const uint4*>(a.xpre);
        uint4* dst = reinterpret_cast<uint4*>(xq);
        for (int base = threadIdx.x; base < n16; base += 8 * MT_NC * 32) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int t = base + j * MT_NC * 32;
                v[j] = t < n16 ? __ldcg(src + t) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int t = base + j * MT_NC * 32;
                if (t < n16) dst[t] = v[j];
            }
        }
    } else if (rms1) {
        mt_quantise_x_rms<F::S16, MT_NC>(a, K, xq, threadIdx.x, red, nwr, a.tp.in_call >= 0 ? &a.tp : nullptr, ep_in);
    } else {
        const float rs = a.xmode == MV_X_RMSNORM ? mt_rms_scale<MT_NC>(a.x, K, a.eps, red, threadIdx.x) : 1.f;
        mt_quantise_x<F::S16>(a, K, xq, threadIdx.x, MT_NC * 32, rs);
    }
    mt_consumer_sync<MT_NC>();
    MtLane L4, L6;   // fragment maps of the Q4_K and Q6_K stage consumers
    L4.gq = L6.gq = lane >> 2;
    L4.c = L6.c = lane & 3;
    const bool bact = L4.c == (L4.gq >> 1);   // this lane carries a nonzero B fragment
    const bool b2act = bact && !(L4.gq & 1);   // column 2c of the third-limb MMA
    L4.xlb = bact ? xq + (L4.gq & 1) * K + MtQ4K::XB_LANE * L4.c : smem + zero_off;
    L6.xlb = bact ? xq + (L6.gq & 1) * K + MtQ6K::XB_LANE * L6.c : smem + zero_off;
    L4.xstr = L6.xstr = bact ? 256 : 0;
    L4.x2b = b2act ? xq + 2 * K + MtQ4K::XB_LANE * L4.c : smem + zero_off;
    L6.x2b = b2act ? xq + 2 * K + MtQ6K::XB_LANE * L6.c : smem + zero_off;
    L4.x2str = L6.x2str = b2act ? 256 : 0;
    int gi = 0;
    bool ok = true;
    float acc_a[2] = {0.f, 0.f}, acc_b[2] = {0.f, 0.f};
    // item t's matrix, group and item within the group (the producer's walk),
    // its ring slot and barrier parity: advanced per stage without divisions
    int m, grp, it;
    mt_locate(a, t0, m, grp, it);
    int s = 0;
    unsigned ph = 0;
    for (int t = t0; t < t1;) {
        if (ok) ok = mbs_wait(bar_full + 8 * s, ph, &g_gb_device_err);
        if (ok) {
            const bool q6 = MIXED ? a.fmt[m] != 0 : FQ6;
            if (q6)
                MtQ6K::consume(smem + s * F::STG, it * MtQ6K::IG, min(nb, (it + 1) * MtQ6K::IG), warp, L6, xq, K,
                               acc_a, acc_b);
            else
                MtQ4K::consume(smem + s * F::STG, it * MtQ4K::IG, min(nb, (it + 1) * MtQ4K::IG), warp, L4, xq, K,
                               acc_a, acc_b);
        }
        __syncwarp();
        if (lane == 0) mbs_arrive(bar_empty + 8 * s);
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
        t++;

        const int nch = a.nchm[m];
        if (it + 1 == nch || t == t1) {   // ---- this CTA's part of group grp of matrix m is done
            const int gl = a.gbase[m] + grp;   // the launch's group index (tickets)
            const int gq = L4.gq, c = L4.c;
#pragma unroll
            for (int j = 0; j < 2; j++) {   // the two 16-row tiles
                acc_a[j] += __shfl_xor_sync(0xffffffffu, acc_a[j], 1);
                acc_a[j] += __shfl_xor_sync(0xffffffffu, acc_a[j], 2);
                acc_b[j] += __shfl_xor_sync(0xffffffffu, acc_b[j], 1);
                acc_b[j] += __shfl_xor_sync(0xffffffffu, acc_b[j], 2);
            }
            const int slot = gi % NSLOT;
            float* rs = red + (slot * MT_NC + warp) * MT_GR;
            if (c == 0) {
                rs[gq] = acc_a[0];
                rs[gq + 8] = acc_b[0];
                rs[16 + gq] = acc_a[1];
                rs[24 + gq] = acc_b[1];
            }
            __syncwarp();
            unsigned tk = 0;
            if (lane == 0) {
                __threadfence_block();
                tk = atomicAdd(&cnt[slot], 1u);
            }
            tk = __shfl_sync(0xffffffffu, tk, 0);
            if (tk == MT_NC - 1) {   // last consumer warp: sum the CTA's partials in warp order
                __threadfence_block();
                float v = 0.f;
                const float* r0 = red + slot * MT_NC * MT_GR + lane;
#pragma unroll
                for (int w2 = 0; w2 < MT_NC; w2++) v += r0[w2 * MT_GR];
                __syncwarp();
                if (lane == 0) cnt[slot] = 0;
                const int gs = a.swq_out ? 2 * grp + m : a.ibase[m] + grp * nch;   // the group's first item
                const int row = grp * MT_GR + lane;
                const float* const rm = a.residual[m];
                if (gs >= t0 && gs + nch <= t1) {
                    if (row < a.rows[m]) mt_put(a, m, row, v + (rm ? rm[row] : 0.f), ep_push);
                    if (a.swq_out) {   // SwiGLU product of pair grp, quantised for ffn_down
                        const float val = row < a.rows[m] ? v : 0.f;
                        float gate = 0.f, up = 0.f;
                        bool have = false;
                        if (m == 0 && gs + 1 < t1) {           // the up half follows in this CTA
                            stash[(grp & 1) * MT_GR + lane] = val;
                        } else if (m == 1 && gs - 1 >= t0) {   // the gate half was this CTA's
                            gate = stash[(grp & 1) * MT_GR + lane];
                            up = val;
                            have = true;
                        } else {   // halves in two CTAs: the second to finish pairs them
                            // one release for the warp's y rows (warp barrier, then
                            // lane 0 fences at GPU scope and takes the pair's
                            // ticket with an acquire-release atomic); the warp
                            // barrier after it orders the lanes' reads behind the
                            // acquire
                            __syncwarp();
                            unsigned k = 0;
                            if (lane == 0) {
                                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                                k = atom_add_acq_rel(&a.swq_tk[grp], 1u);
                            }
                            k = __shfl_sync(0xffffffffu, k, 0);
                            __syncwarp();
                            if (k == 1u) {
                                const float oth = row < a.rows[1 - m] ? __ldcg(a.y[1 - m] + row) : 0.f;
                                gate = m == 0 ? val : oth;
                                up = m == 0 ? oth : val;
                                have = true;
                                if (lane == 0) a.swq_tk[grp] = 0u;
                            }
                        }
                        if (have) mt_quantise32(a.swq_out, a.swq_K, grp, lane, mt_silu_mul(gate, up));
                    }
                } else {
                    // split group: every owner publishes its partial rows and
                    // takes a ticket; the last one sums the partials in CTA
                    // order (deterministic).  Wait-free: no CTA waits on
                    // another, so launches on concurrent streams cannot block
                    // each other.
                    const int half = t0 >= gs ? 0 : 1;   // the group is this CTA's first
                    a.part[(c0 * 2 + half) * MT_GR + lane] = v;
                    __syncwarp();
                    const int cf = mt_owner(gs, a.T, a.ncta), cl2 = mt_owner(gs + nch - 1, a.T, a.ncta);   // unit == 1 here
                    unsigned g = 0;
                    if (lane == 0) g = atom_add_acq_rel(&a.tickets[gl], 1u);
                    g = __shfl_sync(0xffffffffu, g, 0);
                    __syncwarp();
                    if (g == (unsigned)(cl2 - cf)) {
                        float u = 0.f;
                        for (int c2 = cf; c2 <= cl2; c2++) {
                            const int h2 = mt_start(c2, a.T, a.ncta) >= gs ? 0 : 1;
                            u += __ldcg(a.part + (c2 * 2 + h2) * MT_GR + lane);
                        }
                        if (row < a.rows[m]) mt_put(a, m, row, u + (rm ? rm[row] : 0.f), ep_push);
                        if (lane == 0) a.tickets[gl] = 0u;
                    }
                }
            }
            acc_a[0] = acc_a[1] = acc_b[0] = acc_b[1] = 0.f;
            gi++;
        }
        if (++it == nch) {   // the next item starts a group
            it = 0;
            if (a.swq_out) {   // gate g, up g, gate g + 1, ...
                if (m) {
                    m = 0;
                    grp++;
                } else {
                    m = 1;
                }
            } else if (t == a.ibase[m + 1]) {
                m++;
                grp = 0;
            } else {
                grp++;
            }
        }
    }
}

// ================================================================== launch
__host__ __device__ constexpr int round_up(int v, int a) { return (v + a - 1) / a * a; }

static int staged_bytes(int dtype, int nb) {
    switch (dtype) {
        case GB_DT_Q4_K: return nb * (64 * 8 + 16 * 4 + 32 * 8);
        case GB_DT_Q6_K: return nb * (64 * 8 + 48 * 4 + 32 * 8);
        case GB_DT_Q5_K: return nb * 256 * 4 + nb * 32 * 4;   // x fp32 + sums of 8 columns
        case GB_DT_F16: return nb * 32 * 4;
        default: return ((nb + 7) / 8) * 32 * (2 * 16 + 4);
    }
}

// Geometry: 16-row groups; the sub-tile width KC (a multiple of 8 blocks, or
// the whole row when shorter) is the largest that leaves >= 4 ring stages
// (>= 3 for very long rows).
static bool choose_geom(int dtype, int rows, int nb, MvGeom* g) {
    const int bytes = (int)gb_block_bytes(dtype);
    const int xb = round_up(staged_bytes(dtype, nb), 128);
    g->T = 16;
    const int red = round_up(10 * MV_CONSUMERS * g->T * 4, 128);   // S + 2 <= 10 slots
    const long avail = MV_SMEM_MAX - xb - red - 256;
    int kc_best = 0;
    for (int min_stages = 4; min_stages >= 2 && !kc_best; min_stages--) {
        for (int KC = nb; KC >= 1; KC = KC > 8 ? ((KC - 1) & ~7) : KC - 1) {
            if (KC < nb && (KC & 7)) continue;
            const int RS = round_up(KC * bytes + 32, 128) + 16;
            const long SB = (long)g->T * RS + 128;
            if (SB * min_stages <= avail) { kc_best = KC; break; }
        }
    }
    if (!kc_best) return false;
    g->KC = kc_best;
    g->nk = (nb + g->KC - 1) / g->KC;
    g->RS = round_up(g->KC * bytes + 32, 128) + 16;
    g->SB = g->T * g->RS + 128;
    g->ngroups = (rows + g->T - 1) / g->T;
    g->red_off = xb;
    g->ring_off = xb + red;
    const int S = (int)((MV_SMEM_MAX - g->ring_off - 256) / g->SB);
    g->S = S > 8 ? 8 : S;
    g->bar_off = g->ring_off + g->S * g->SB;
    return g->S >= 2;
}

template <typename K>
static cudaError_t launch_kernel(K kernel, const void* W, int rows, int nb, const float* x, float* y,
                                 const float* residual, const MvGeom& g, cudaStream_t st) {
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(kernel), MV_SMEM_MAX);
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)g.bar_off + 2 * g.S * sizeof(uint64_t) + (g.S + 3) * sizeof(int);
    const int nsm = sm_count();
    const int grid = g.ngroups < nsm ? g.ngroups : nsm;
    kernel<<<grid, MV_THREADS, smem, st>>>(static_cast<const uint8_t*>(W), rows, nb, x, y, residual, g);
    return cudaGetLastError();
}

}  // namespace gb

using namespace gb;

namespace gb {

// ------------------------------------------------------------------ plans
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tensor map of the 3-D view {box row as u64, rows, z} of a Q4_K (z = block,
// box depth boxz blocks) or Q6_K (z = 8-block run, depth 1) matrix with nb
// blocks per row.  W and the row pitch must be 16-byte aligned.
bool mt_encode_view(void* map128, int dtype, const void* W, int rows, int nb, int boxz) {
    auto enc = tensor_map_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(W) & 15)) return false;
    const bool q6 = dtype == GB_DT_Q6_K;
    if (!q6 && dtype != GB_DT_Q4_K) return false;
    if (q6 && (nb % 8 || boxz != 1)) return false;
    const int blk = q6 ? GB_Q6K_BYTES : GB_Q4K_BYTES;
    const int inner = (q6 ? 8 : 1) * blk;
    cuuint64_t dims[3] = {(cuuint64_t)inner / 8, (cuuint64_t)rows, (cuuint64_t)(nb / (q6 ? 8 : 1))};
    cuuint64_t strides[2] = {(cuuint64_t)nb * blk, (cuuint64_t)inner};
    cuuint32_t box[3] = {(cuuint32_t)inner / 8, MT_GR, (cuuint32_t)boxz};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(W), dims,
               strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of a Q4_K matrix as rows of bytes {18 nb u64, rows, 1}: a box
// {box_u64, 32 rows} copies box_u64 * 8 consecutive bytes of 32 rows (x
// coordinates are multiples of 18 u64 = one block, 16-byte aligned; bytes past
// the row end are zero-filled).
bool mt_encode_rows(void* map128, const void* W, int rows, int nb, int box_u64) {
    auto enc = tensor_map_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(W) & 15) || box_u64 <= 0 || box_u64 > 256 || box_u64 % 2) return false;
    const cuuint64_t rb = (cuuint64_t)nb * GB_Q4K_BYTES;
    cuuint64_t dims[3] = {rb / 8, (cuuint64_t)rows, 1};
    cuuint64_t strides[2] = {rb, rb * (cuuint64_t)rows};
    cuuint32_t box[3] = {(cuuint32_t)box_u64, MT_GR, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(W), dims,
               strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_encode_x(void* map128, const float* X, int T, int K, int box_k, int box_t) {
    auto enc = tensor_map_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(X) & 15) || K % 4 || box_k * 4 % 16) return false;
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)T, 1};
    cuuint64_t strides[2] = {(cuuint64_t)K * 4, (cuuint64_t)K * 4 * (cuuint64_t)T};
    cuuint32_t box[3] = {(cuuint32_t)box_k, (cuuint32_t)box_t, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(X), dims,
               strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Split fp16 activations laid out column-group-major, [K / 8][Tp][8 halves]
// (Tp a multiple of 256), viewed as {256 x u64 = 128 rows of one group, Tp /
// 128, K / 8}: a box {256, box_t / 128, 4} copies 2 KB runs and lands as the
// tensor cores' K-major tile of box_t rows x 32 columns (core matrices of 8
// rows x 16 bytes, column groups box_t x 16 bytes apart).
bool gemm_encode_x16(void* map128, const void* X16, int Tp, int K, int box_t) {
    auto enc = tensor_map_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(X16) & 15) || K % 32 || Tp % 256 || box_t % 128) return false;
    cuuint64_t dims[3] = {256, (cuuint64_t)Tp / 128, (cuuint64_t)K / 8};
    cuuint64_t strides[2] = {2048, (cuuint64_t)Tp * 16};
    cuuint32_t box[3] = {256, (cuuint32_t)box_t / 128, 4};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(X16), dims,
               strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <class F>
static size_t mt_smem_bytes(int S, int K) {
    const size_t xq = ((size_t)mt_xq_bytes(K, F::S16) + 15) & ~(size_t)15;
    const int nslot = S + 2;
    return (size_t)S * F::STG + xq + MT_ZERO + (size_t)nslot * F::NC * MT_GR * 4 + (size_t)nslot * 4 + 16 +
           16 * (size_t)S + 16 + 2 * MT_GR * 4;   // + the SwiGLU stash
}

// Encode the 3-D view {one box row of bytes as u64, rows, z} of W for format F.
template <class F>
static bool mt_encode(MvPlan* p, const void* W, int rows, int nb) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    int S = 4;
    while (S > 2 && mt_smem_bytes<F>(S, nb * 256) > (size_t)MV_SMEM_MAX) S--;
    if (mt_smem_bytes<F>(S, nb * 256) > (size_t)MV_SMEM_MAX) return false;
    const int blk = F::STG / (MT_GR * F::KC);   // bytes per block
    const cuuint64_t rb = (cuuint64_t)nb * blk;
    const int inner = F::ZUNIT * blk;   // bytes per box row
    cuuint64_t dims[3] = {(cuuint64_t)inner / 8, (cuuint64_t)rows, (cuuint64_t)(nb / F::ZUNIT)};
    cuuint64_t strides[2] = {rb, (cuuint64_t)inner};
    cuuint32_t box[3] = {(cuuint32_t)inner / 8, MT_GR, (cuuint32_t)F::BOXZ};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(reinterpret_cast<CUtensorMap*>(p->tmap), CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(W), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    p->kind = MV_TMA;
    p->S = S;
    p->smem = mt_smem_bytes<F>(S, nb * 256);
    p->nch = (nb + F::IG - 1) / F::IG;   // split items per 32-row group
    p->ngroups = (rows + MT_GR - 1) / MT_GR;
    p->T = p->ngroups * p->nch;
    p->ncta = std::min(p->T, sm_count());
    return true;
}

int mv_plan(MvPlan* p, int dtype, const void* W, int rows, int cols) {
    if (!p || !W || rows <= 0 || cols <= 0) return GB_EINVAL;
    if (reinterpret_cast<uintptr_t>(W) & 15) return GB_EINVAL;
    if (dtype != GB_DT_Q4_K && dtype != GB_DT_Q6_K && dtype != GB_DT_Q8_0 && dtype != GB_DT_Q5_K &&
        dtype != GB_DT_F16)
        return GB_EINVAL;
    const int width = gb_block_width(dtype);
    if (cols % width) return GB_ESHAPE;
    *p = MvPlan{};
    p->W = W;
    p->dtype = dtype;
    p->rows = rows;
    p->cols = cols;
    p->nb = cols / width;
    p->kind = MV_RING;
    // TMA path: Q4_K rows (144 nb bytes) are always 16-byte multiples; Q6_K
    // rows (210 nb bytes) are when nb is a multiple of 8.
    if (dtype == GB_DT_Q4_K) mt_encode<MtQ4K>(p, W, rows, p->nb);
    if (dtype == GB_DT_Q6_K && p->nb % 8 == 0) mt_encode<MtQ6K>(p, W, rows, p->nb);
    if (p->kind == MV_RING) {
        MvGeom g;
        if (!choose_geom(dtype, rows, p->nb, &g)) return GB_ELIMIT;
    }
    return GB_OK;
}

size_t mv_ws_bytes(const MvPlan& p) {
    if (p.kind != MV_TMA) return 0;
    return (size_t)GB_MAX_SMS * 2 * MT_GR * sizeof(float) + ((size_t)p.ngroups * sizeof(unsigned) + 255) / 256 * 256;
}

// Matvec launches carry the programmatic-dependent-launch attribute: after a
// predecessor that has executed griddepcontrol.launch_dependents (the matvec
// and attention kernels do so at their top) the CTAs start at once and stream
// weight boxes; they read x, the residual and the workspace and write y only
// after griddepcontrol.wait (the predecessor complete and its writes visible).
// After any other predecessor the launch behaves as a plain one.  Weights must
// therefore not be written by a kernel that triggers its dependents early (no
// kernel of this library writes weights).
// GB_DISABLE_PDL=1 in the environment turns programmatic dependent launch off
// (every matvec then waits for the previous kernel to finish before starting).
static bool pdl_allowed() {
    static const bool ok = [] {
        const char* e = getenv("GB_DISABLE_PDL");
        return !(e && e[0] && e[0] != '0');
    }();
    return ok;
}

// GB_MV_L2PF=k in the environment: at its start, once its ring is full,
// each CTA also prefetches its next k boxes into L2.
static int mv_l2_prefetch() {
    static const int v = [] {
        const char* e = getenv("GB_MV_L2PF");
        return e ? atoi(e) : 0;
    }();
    return v;
}

static int mv_check_xform(const MvXform* xf, bool tma) {
    const int xmode = xf ? xf->mode : MV_X_NONE;
    if (xf && (xf->swq_out || xf->swq_tk) && !tma) return GB_EINVAL;
    if (xmode == MV_X_NONE) return GB_OK;
    if (!tma) return GB_EINVAL;   // transforms run in the TMA kernels' x quantiser only
    if (xmode == MV_X_PREQ) return xf->xq && !(reinterpret_cast<uintptr_t>(xf->xq) & 15) ? GB_OK : GB_EINVAL;
    const float* other = xmode == MV_X_RMSNORM ? xf->w : xf->x2;
    if (!other || (reinterpret_cast<uintptr_t>(other) & 15)) return GB_EINVAL;
    return GB_OK;
}

int mv_launch(const MvPlan& p, const float* x, float* y, const float* residual, void* ws, cudaStream_t st, bool pdl,
              const MvXform* xf, const MvTp* tp) {
    if (!x || !y) return GB_EINVAL;
    if (reinterpret_cast<uintptr_t>(x) & 15) return GB_EINVAL;
    if (p.kind == MV_TMA) {
        const MvPlan* ps[1] = {&p};
        float* ys[1] = {y};
        const float* rs[1] = {residual};
        return mv_launch_group(ps, 1, x, ys, rs, ws, st, pdl, xf, tp);
    }
    if (tp && (tp->push_call >= 0 || tp->in_call >= 0)) return GB_EINVAL;   // exchanges run in the TMA kernels only
    int rc = mv_check_xform(xf, false);
    if (rc) return rc;
    MvGeom g;
    if (!choose_geom(p.dtype, p.rows, p.nb, &g)) return GB_ELIMIT;
    cudaError_t e;
    switch (p.dtype) {
        case GB_DT_Q4_K: e = launch_kernel(k_mv_q4k, p.W, p.rows, p.nb, x, y, residual, g, st); break;
        case GB_DT_Q6_K: e = launch_kernel(k_mv_q6k, p.W, p.rows, p.nb, x, y, residual, g, st); break;
        case GB_DT_Q5_K: e = launch_kernel(k_mv_plain<GB_DT_Q5_K>, p.W, p.rows, p.nb, x, y, residual, g, st); break;
        case GB_DT_F16: e = launch_kernel(k_mv_plain<GB_DT_F16>, p.W, p.rows, p.nb, x, y, residual, g, st); break;
        default: e = launch_kernel(k_mv_q8_0, p.W, p.rows, p.nb, x, y, residual, g, st); break;
    }
    return e == cudaSuccess ? GB_OK : GB_ECUDA;
}

size_t mv_ws_bytes_group(const MvPlan* const* ps, int n) {
    if (!mv_groupable(ps, n)) return 0;
    size_t groups = 0;
    for (int i = 0; i < n; i++) groups += (size_t)ps[i]->ngroups;
    return (size_t)GB_MAX_SMS * 2 * MT_GR * sizeof(float) + (groups * sizeof(unsigned) + 255) / 256 * 256;
}

// Ring depth of a mixed-format launch with K columns (0 if none fits).
static int mix_stages(int K) {
    for (int S = 4; S >= 2; S--)
        if (mt_smem_bytes<MtMix>(S, K) <= (size_t)MV_SMEM_MAX) return S;
    return 0;
}

template <class F>
static cudaError_t mvt_configure() {
    return set_smem_once(reinterpret_cast<const void*>(k_mvt<F>), MV_SMEM_MAX);
}

int mv_launch_group(const MvPlan* const* ps, int n, const float* x, float* const* ys, const float* const* res,
                    void* ws, cudaStream_t st, bool pdl, const MvXform* xf, const MvTp* tp) {
    if (!x || !ys || !mv_groupable(ps, n)) return GB_EINVAL;
    if (reinterpret_cast<uintptr_t>(x) & 15) return GB_EINVAL;
    int rc = mv_check_xform(xf, true);
    if (rc) return rc;
    const MvPlan& p = *ps[0];
    bool mixed = false;
    for (int i = 1; i < n; i++) mixed |= ps[i]->dtype != p.dtype;
    if (mixed) {   // matrices with more items per group first (their groups get whole CTAs)
        int ord[MT_MAXM];
        for (int i = 0; i < n; i++) ord[i] = i;
        std::stable_sort(ord, ord + n, [&](int u, int v) { return ps[u]->nch > ps[v]->nch; });
        bool moved = false;
        for (int i = 0; i < n; i++) moved |= ord[i] != i;
        if (moved) {
            const MvPlan* ps2[MT_MAXM];
            float* ys2[MT_MAXM];
            const float* rs2[MT_MAXM];
            for (int i = 0; i < n; i++) {
                ps2[i] = ps[ord[i]];
                ys2[i] = ys[ord[i]];
                rs2[i] = res ? res[ord[i]] : nullptr;
            }
            return mv_launch_group(ps2, n, x, ys2, rs2, ws, st, pdl, xf, tp);
        }
    }
    if (mixed && !ws) {   // mixed formats split by items, which needs the workspace: one launch per matrix
        for (int i = 0; i < n; i++)
            if ((rc = mv_launch_group(&ps[i], 1, x, &ys[i], res ? &res[i] : nullptr, ws, st, pdl, xf, tp))) return rc;
        return GB_OK;
    }
    if (tp && (tp->push_call >= 0 || tp->in_call >= 0)) {   // tensor-parallel exchange: check its shape
        if (!tp->peers || !tp->step || !tp->err || tp->world < 2 || tp->H <= 0) return GB_EINVAL;
        if (tp->push_call >= 0 && (n != 1 || (res && res[0]) || ps[0]->rows > tp->H)) return GB_EINVAL;
        if (tp->in_call >= 0 && (!xf || xf->mode != MV_X_RMSNORM || p.nb * 256 != tp->H ||
                                 p.nb * 64 > MT_XU * MtMix::NC * 32 || !tp->h_out ||
                                 (reinterpret_cast<uintptr_t>(tp->h_out) & 15)))
            return GB_EINVAL;
    }
    const bool q6 = p.dtype == GB_DT_Q6_K;
    GB_CUDA_TRY(mixed ? mvt_configure<MtMix>() : (q6 ? mvt_configure<MtQ6K>() : mvt_configure<MtQ4K>()));
    MtArgs a = {};
    a.x = x;
    a.nm = n;
    a.gbase[0] = 0;
    a.ibase[0] = 0;
    for (int i = 0; i < MT_MAXM; i++) {
        const bool on = i < n;
        if (on && !ys[i]) return GB_EINVAL;
        a.y[i] = on ? ys[i] : nullptr;
        a.residual[i] = on && res ? res[i] : nullptr;
        a.rows[i] = on ? ps[i]->rows : 0;
        a.nchm[i] = on ? ps[i]->nch : 1;
        a.fmt[i] = on && ps[i]->dtype == GB_DT_Q6_K ? 1 : 0;
        a.gbase[i + 1] = a.gbase[i] + (on ? ps[i]->ngroups : 0);
        a.ibase[i + 1] = a.ibase[i] + (on ? ps[i]->ngroups * ps[i]->nch : 0);
    }
    const int groups = a.gbase[MT_MAXM];
    a.part = static_cast<float*>(ws);
    a.tickets = ws ? reinterpret_cast<unsigned*>(static_cast<char*>(ws) + (size_t)GB_MAX_SMS * 2 * MT_GR * sizeof(float))
                   : nullptr;
    a.nb = p.nb;
    a.T = a.ibase[MT_MAXM];
    a.xmode = xf ? xf->mode : MV_X_NONE;
    a.nw = a.xmode == MV_X_RMSNORM ? xf->w : nullptr;
    a.x2 = a.xmode == MV_X_SILU_MUL ? xf->x2 : nullptr;
    a.eps = xf ? xf->eps : 0.f;
    a.xpre = a.xmode == MV_X_PREQ ? xf->xq : nullptr;
    if (xf && xf->swq_out) {   // gate / up: two matrices of equal rows, one item per group
        const int kq = xf->swq_K ? xf->swq_K : ps[0]->rows;
        if (n != 2 || mixed || p.nch != 1 || ps[1]->nch != 1 || ps[0]->rows != ps[1]->rows || !xf->swq_tk ||
            (res && (res[0] || res[1])) || kq % 256 || kq < ps[0]->rows || (tp && tp->push_call >= 0))
            return GB_EINVAL;
        a.swq_out = xf->swq_out;
        a.swq_tk = xf->swq_tk;
        a.swq_K = kq;
    }
    if (tp) a.tp = *tp;
    if (!tp) a.tp.push_call = a.tp.in_call = -1;
    // with a workspace: stream-K over items; without: whole groups per CTA
    // (one format, so every group has the same item count).  Whole groups
    // also when they give no CTA more than one item above what stream-K
    // would (e.g. 128 groups of 7 items on 148 SMs): no group is then split,
    // so no CTA ends with the cross-CTA fix-up, which costs more than an item.
    const int nsm = sm_count();
    bool whole = !ws;
    if (ws && !mixed && p.nch > 1)
        whole = (groups + nsm - 1) / nsm * p.nch <= (a.T + nsm - 1) / nsm + 1;
    a.unit = whole ? p.nch : 1;
    const int units = whole ? groups : a.T;
    a.ncta = units < nsm ? units : nsm;
    if (mixed) {   // whole groups of the leading multi-item matrices, one per CTA, when no CTA gets more items
        int g1 = 0, n1 = 0, i = 0;
        for (; i < n && ps[i]->nch > 1; i++) {
            if (n1 && ps[i]->nch != n1) break;
            n1 = ps[i]->nch;
            g1 += ps[i]->ngroups;
        }
        bool rest1 = i < n;
        for (int j = i; j < n; j++) rest1 &= ps[j]->nch == 1;
        const int t2 = a.T - g1 * n1, c2 = nsm - g1;
        if (rest1 && g1 > 0 && c2 > 0 && t2 > 0 &&
            (t2 + c2 - 1) / c2 <= std::max(n1, (a.T + nsm - 1) / nsm)) {
            a.c1 = g1;
            a.n1 = n1;
            a.ncta = g1 + std::min(c2, t2);
        }
    }
    a.S = mixed ? mix_stages(p.nb * 256) : p.S;
    a.l2pf = mv_l2_prefetch();
    if (a.S < 2) return GB_ELIMIT;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ncta);
    cfg.blockDim = dim3((MtMix::NC + 1) * 32);
    cfg.dynamicSmemBytes = mixed ? mt_smem_bytes<MtMix>(a.S, p.nb * 256) : p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && pdl_allowed()) ? 1 : 0;
    const CUtensorMap* m0 = reinterpret_cast<const CUtensorMap*>(ps[0]->tmap);
    const CUtensorMap* m1 = reinterpret_cast<const CUtensorMap*>(ps[n > 1 ? 1 : 0]->tmap);
    const CUtensorMap* m2 = reinterpret_cast<const CUtensorMap*>(ps[n > 2 ? 2 : 0]->tmap);
    if (mixed)
        GB_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_mvt<MtMix>, *m0, *m1, *m2, a));
    else if (q6)
        GB_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_mvt<MtQ6K>, *m0, *m1, *m2, a));
    else
        GB_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_mvt<MtQ4K>, *m0, *m1, *m2, a));
    return GB_OK;
}
// TMA plans of one column count; one format, or Q4_K and Q6_K mixed when a
// ring of at least two mixed stages fits.
bool mv_groupable(const MvPlan* const* ps, int n) {
    if (n < 1 || n > MT_MAXM) return false;
    bool mixed = false;
    for (int i = 0; i < n; i++) {
        if (ps[i]->kind != MV_TMA || ps[i]->nb != ps[0]->nb) return false;
        if (ps[i]->dtype != ps[0]->dtype) mixed = true;
        else if (ps[i]->S != ps[0]->S) return false;
    }
    return !mixed || mix_stages(ps[0]->nb * 256) >= 2;
}

// Workspace for the plain C entry point: one zeroed buffer per (device,
// stream), grown on demand.  Calls on one stream are ordered, so they can
// share it; different streams get different buffers.
static std::mutex g_ws_mu;
static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_ws;

// Returns nullptr when no buffer can be made now (the stream is being
// captured); the launch then splits by whole groups and needs none.
static void* stream_workspace(cudaStream_t st, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_ws_mu);
    auto& e = g_ws[{dev, st}];
    if (e.second >= bytes) return e.first;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
    if (e.first) {
        cudaStreamSynchronize(st);
        cudaFree(e.first);
        e = {nullptr, 0};
    }
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, bytes) != cudaSuccess) return nullptr;
    if (cudaMemsetAsync(ptr, 0, bytes, st) != cudaSuccess) {
        cudaFree(ptr);
        return nullptr;
    }
    e = {ptr, bytes};
    return ptr;
}

}  // namespace gb

extern "C" int gb_matvec(int dtype, const void* W, int rows, int cols, const float* x, float* y,
                         const float* residual, void* stream) {
    if (!W || !x || !y || rows <= 0 || cols <= 0) return GB_EINVAL;
    // Weights are fetched by bulk / tensor copies (16-byte aligned source) and
    // x is read with 128-bit loads.
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return GB_EINVAL;
    MvPlan p;
    int rc = mv_plan(&p, dtype, W, rows, cols);
    if (rc) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* ws = p.kind == MV_TMA ? stream_workspace(st, mv_ws_bytes(p)) : nullptr;
    return mv_launch(p, x, y, residual, ws, st, true, nullptr);
}

extern "C" int gb_matvec_group(int n, const int* dtypes, const void* const* W, const int* rows, int cols,
                               const float* x, float* const* y, void* stream) {
    if (n < 1 || n > MT_MAXM || !dtypes || !W || !rows || !x || !y || cols <= 0) return GB_EINVAL;
    if (reinterpret_cast<uintptr_t>(x) & 15) return GB_EINVAL;
    MvPlan plans[MT_MAXM];
    const MvPlan* ps[MT_MAXM];
    for (int i = 0; i < n; i++) {
        if (!W[i] || !y[i] || rows[i] <= 0 || (reinterpret_cast<uintptr_t>(W[i]) & 15)) return GB_EINVAL;
        const int rc = mv_plan(&plans[i], dtypes[i], W[i], rows[i], cols);
        if (rc) return rc;
        ps[i] = &plans[i];
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (mv_groupable(ps, n)) {
        void* ws = stream_workspace(st, mv_ws_bytes_group(ps, n));
        return mv_launch_group(ps, n, x, y, nullptr, ws, st, true, nullptr);
    }
    for (int i = 0; i < n; i++) {
        void* ws = plans[i].kind == MV_TMA ? stream_workspace(st, mv_ws_bytes(plans[i])) : nullptr;
        const int rc = mv_launch(plans[i], x, y[i], nullptr, ws, st, true, nullptr);
        if (rc) return rc;
    }
    return GB_OK;
}

extern "C" int gb_device_error(int clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gb_device_err, sizeof(v)) != cudaSuccess) return GB_ECUDA;
    if (clear && v) {
        const unsigned z = 0;
        if (cudaMemcpyToSymbol(g_gb_device_err, &z, sizeof(z)) != cudaSuccess) return GB_ECUDA;
    }
    return -(int)v;
}
