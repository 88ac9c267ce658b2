// gb_mt.cuh -- device building blocks of the TMA-fed tensor-core matvec
// (gb_matvec.cu), also used by the attention kernel to quantise its output
// for the next matvec.
#pragma once
#include "gb_common.cuh"
#include "gb_internal.h"

#include <cuda.h>

namespace gb {

constexpr unsigned long long MT_WAIT_NS = 2000000000ull;   // bound on every wait (2 s)

// ------------------------------------------------------------------ primitives
__device__ __forceinline__ uint32_t sptr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// D += A(16x32 u8, row) * B(32x8 s8, col), s32 accumulate.
__device__ __forceinline__ void mma_u8s8(int4& d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d.x), "+r"(d.y), "+r"(d.z), "+r"(d.w)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Three int8 limbs of x: x ~ s (x0 + x1 / 256 + x2 / 65536), |x0| <= 127,
// s = max|x| / 127 over the 32-column sub-block; v is x / s.  Every step is
// exact in fp32 (v - x0, the scalings by 256, t - rint(t)), so the limbs
// carry v to 2^-17 (24 significant bits at the sub-block's maximum): x enters
// the int8 tensor cores at fp32 precision.  A middle limb that rounds to 128
// moves one unit into x0 (x0 <= 126 then), so it stays in int8.
__device__ __forceinline__ void limbs(float v, int& x0, int& x1, int& x2) {
    const float r0 = rintf(v);
    const float t1 = (v - r0) * 256.f;
    const float r1 = rintf(t1);
    const int r2 = (int)rintf((t1 - r1) * 256.f);
    x0 = (int)r0;
    x1 = (int)r1;
    if (x1 > 127) {   // 128 / 256 = 1 - 128 / 256
        x1 -= 256;
        x0 += 1;
    }
    x2 = r2 > 127 ? 127 : (r2 < -128 ? -128 : r2);
}
// The value a limb triple stands for, in units of the sub-block scale s
// (exact: 24 bits).
__device__ __forceinline__ float limb_value(int x0, int x1, int x2) {
    return fmaf((float)x2, 1.0f / 65536.0f, fmaf((float)x1, 0.00390625f, (float)x0));
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}

// ================================================================== TMA path
// Weights stream through a ring of shared-memory stages filled by TMA tensor
// copies.  Q4_K: the matrix is viewed as a 3-D tensor {144-byte block
// (18 x u64), row, block index} with strides {row_bytes, 144}; one box
// {18, 32 rows, 1 block} is one split item, and up to 16 of them (consecutive
// blocks of one 32-row group) fill a stage laid out [block][row][144 B], so
// every 16-row tile of a block is a dense 2304-byte slab (conflict-free
// 128-bit reads).  Q6_K: the item is a run of 8 blocks (1680 bytes, the
// shortest 16-byte multiple) of 32 rows.  Every copy starts at x = 0 (16-byte
// aligned).  Out-of-range rows are zero-filled by the TMA unit and skipped.
//
// Work split (stream-K): the (32-row group, item) sequence is cut into one
// contiguous range per CTA, so every CTA streams the same number of bytes
// to within one item.  Groups that straddle CTAs finish through a per-group
// ticket: each owner writes its partial rows to the workspace and the last
// one sums the partials in CTA order (deterministic) and writes y.
//
// x is quantised inside every CTA (int8 limb planes + per-32-column scale and
// sum in shared memory) while the first weight boxes are in flight.  With
// programmatic dependent launch the producer issues those boxes before
// griddepcontrol.wait; consumers read x and write y only after it.
constexpr int MT_GR = 32;                 // rows per group (two 16-row tiles)

__device__ __forceinline__ void mbs_init(uint32_t b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void mbs_expect(uint32_t b, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(tx) : "memory");
}
__device__ __forceinline__ void mbs_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ bool mbs_test(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait (2 s of %globaltimer); false on timeout, recorded as
// GB_ETIMEOUT in the error word *err.
static __device__ __noinline__ bool mbs_wait_slow(uint32_t b, uint32_t parity, unsigned* err) {
    const uint64_t t0 = gtimer();
    while (!mbs_test(b, parity)) {
        if (gtimer() - t0 > MT_WAIT_NS) {
            atomicExch(err, (unsigned)(-GB_ETIMEOUT));
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool mbs_wait(uint32_t b, uint32_t parity, unsigned* err) {
    return mbs_test(b, parity) || mbs_wait_slow(b, parity, err);
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
// L2 prefetch of one tensor-map box (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_3d(const void* map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
template <int NC>
__device__ __forceinline__ void mt_consumer_sync() {
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory");
}
// Split item t of a matrix with nch items per group: CTA c owns
// [t_start(c), t_start(c + 1)); owner(t) is the CTA whose range holds t.
__device__ __forceinline__ int mt_start(int c, int T, int n) { return (int)((long long)c * T / n); }
__device__ __forceinline__ int mt_owner(int t, int T, int n) { return (int)(((long long)(t + 1) * n - 1) / T); }

// x in shared memory (K = 256 nb columns):
//   x0[K], x1[K], x2[K]         int8 limbs, x ~ s (x0 + x1 / 256 + x2 / 65536)
//   f[K/64][4]                  per 64 columns {s lo, s hi, sum lo, sum hi} of
//                               its two 32-column sub-blocks (s = max|x| / 127)
//   s16[K/256][2][8]  (Q6_K)    sums of the 16-column sub-blocks 8n + 2G + h,
//                               stored at [b][h][4n + G]
__host__ __device__ constexpr int mt_xq_bytes(int K, bool s16) { return 3 * K + K / 4 + (s16 ? K / 4 : 0); }
constexpr int MT_ZERO = 256;   // zero line read by lanes without a B fragment

// RMSNorm scale 1 / sqrt(mean(x^2) + eps) over the K columns, summed by the
// consumer threads and combined in fixed warp order (every CTA gets the
// same value).  scratch: NC floats of shared memory.
constexpr int MT_XU = 4;   // float4 loads of x in flight per thread
template <int NC>
__device__ __forceinline__ float mt_rms_scale(const float* __restrict__ x, int K, float eps, float* scratch, int tid) {
    float ss = 0.f;
    const int n4 = K / 4;
    for (int base = tid; base < n4; base += MT_XU * NC * 32) {
        float4 v[MT_XU];
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            const int t = base + j * NC * 32;
            v[j] = t < n4 ? __ldcg(reinterpret_cast<const float4*>(x) + t) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            ss = fmaf(v[j].x, v[j].x, ss);
            ss = fmaf(v[j].y, v[j].y, ss);
            ss = fmaf(v[j].z, v[j].z, ss);
            ss = fmaf(v[j].w, v[j].w, ss);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) scratch[tid >> 5] = ss;
    mt_consumer_sync<NC>();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NC; w++) tot += scratch[w];
    return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
}
// silu(g) u = g u / (1 + e^-g) with the fast exponential and divide (a few
// ulp): x is quantised to ~16 bits right after, far coarser.  g is clamped at
// -80 so 1 + e^-g stays finite (silu(-80) is ~1e-33, zero at x's scale).
__device__ __forceinline__ float mt_silu_mul(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-fmaxf(g, -80.f))) * u;
}

// One float4 of x (columns 4t .. 4t + 3): transform, quantise to three int8
// limbs per value against the 32-column sub-block's max |x|, and record the
// sub-block scale and sum.  Lanes 8k .. 8k + 7 of a warp hold one sub-block.
template <bool S16, class A>
__device__ __forceinline__ void mt_quantise4(const A& a, int K, uint8_t* xq, int t, float4 v, float4 w, float rs) {
    uint32_t* p0 = reinterpret_cast<uint32_t*>(xq);
    uint32_t* p1 = reinterpret_cast<uint32_t*>(xq + K);
    uint32_t* p2 = reinterpret_cast<uint32_t*>(xq + 2 * K);
    float* f = reinterpret_cast<float*>(xq + 3 * K);
    float* f16 = f + K / 16;
    if (a.xmode == MV_X_RMSNORM) {   // w * (x * r), the reference's rounding
        v = make_float4(__fmul_rn(w.x, __fmul_rn(v.x, rs)), __fmul_rn(w.y, __fmul_rn(v.y, rs)),
                        __fmul_rn(w.z, __fmul_rn(v.z, rs)), __fmul_rn(w.w, __fmul_rn(v.w, rs)));
    } else if (a.xmode == MV_X_SILU_MUL) {
        v = make_float4(mt_silu_mul(v.x, w.x), mt_silu_mul(v.y, w.y), mt_silu_mul(v.z, w.z), mt_silu_mul(v.w, w.w));
    }
    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    float sm = (v.x + v.y) + (v.z + v.w);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sm += __shfl_xor_sync(0xffffffffu, sm, o);
    }
    const float inv = mx > 0.f ? 127.f / mx : 0.f;
    int a0, a1, a2, b0, b1, b2, c0, c1, c2, d0, d1, d2;
    limbs(v.x * inv, a0, a1, a2);
    limbs(v.y * inv, b0, b1, b2);
    limbs(v.z * inv, c0, c1, c2);
    limbs(v.w * inv, d0, d1, d2);
    p0[t] = pack4(a0, b0, c0, d0);
    p1[t] = pack4(a1, b1, c1, d1);
    p2[t] = pack4(a2, b2, c2, d2);
    const float s = mx / 127.f;
    if (S16) {
        // 16-column sums of the QUANTISED values s (x0 + x1 / 256): the Q6_K
        // consumer applies the -32 code offset with them, so the offset and
        // the codes multiply the same x, and the quantisation error of x
        // reaches the result only through (q - 32), not through the codes'
        // mean (31.5), which would give every row a correlated error
        float sq = (limb_value(a0, a1, a2) + limb_value(b0, b1, b2)) + (limb_value(c0, c1, c2) + limb_value(d0, d1, d2));
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        if ((t & 3) == 0) {   // 16-column sum: column c0 = 4t = 256 b + 128 n + 32 G + 16 h
            const int cc = 4 * t, b = cc >> 8, n = (cc >> 7) & 1, G = (cc >> 5) & 3, h = (cc >> 4) & 1;
            f16[b * 16 + h * 8 + 4 * n + G] = sq * s;
        }
    }
    const int sb = t >> 3;
    if ((t & 7) == 0) {
        f[(sb >> 1) * 4 + (sb & 1)] = s;
        f[(sb >> 1) * 4 + 2 + (sb & 1)] = sm;
    }
}

// One 32-column sub-block sb of x held one value per lane (lane = column
// 32 sb + lane), quantised by a warp into the x layout above at xq (K
// columns, with the 16-column sums): the same scale, limbs and sums as
// mt_quantise4 computes from float4s.  Used by a matvec that produces the
// next matvec's x (the SwiGLU product of gate / up for ffn_down).
__device__ __forceinline__ void mt_quantise32(uint8_t* xq, int K, int sb, int lane, float v) {
    float mx = fabsf(v), sm = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sm += __shfl_xor_sync(0xffffffffu, sm, o);
    }
    float* f = reinterpret_cast<float*>(xq + 3 * K);
    float* f16 = f + K / 16;
    const float inv = mx > 0.f ? 127.f / mx : 0.f;
    int x0, x1, x2;
    limbs(v * inv, x0, x1, x2);
    xq[32 * sb + lane] = (uint8_t)(x0 & 255);
    xq[K + 32 * sb + lane] = (uint8_t)(x1 & 255);
    xq[2 * K + 32 * sb + lane] = (uint8_t)(x2 & 255);
    const float s = mx / 127.f;
    // 16-column sums of the quantised values (see mt_quantise4)
    float sq = limb_value(x0, x1, x2);
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((lane & 15) == 0) {   // 16-column sum: column c0 = 32 sb + lane = 256 b + 128 n + 32 G + 16 h
        const int c0 = 32 * sb + lane, b = c0 >> 8, n = (c0 >> 7) & 1, G = (c0 >> 5) & 3, h = (c0 >> 4) & 1;
        f16[b * 16 + h * 8 + 4 * n + G] = sq * s;
    }
    if (lane == 0) {
        f[(sb >> 1) * 4 + (sb & 1)] = s;
        f[(sb >> 1) * 4 + 2 + (sb & 1)] = sm;
    }
}

// Quantise x into shared memory.  The loads of MT_XU float4 per thread (and
// of the transform's second operand) are issued before any is used, so the
// L2 latency is paid once per MT_XU float4 rather than once per float4.  x
// is read through L2 (ld.global.cg): in a persistent kernel it was written
// by other CTAs earlier in the same launch.
// nthr is a multiple of 32 and K / 4 of 64, so the bounds test is
// warp-uniform and the shuffles see full warps.
template <bool S16, class A>
__device__ __forceinline__ void mt_quantise_x(const A& a, int K, uint8_t* xq, int tid, int nthr, float rs) {
    const int n4 = K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    const float4* w4 = reinterpret_cast<const float4*>(a.xmode == MV_X_RMSNORM ? a.nw : a.x2);
    const bool aux = a.xmode != MV_X_NONE;
    for (int base = tid; base < n4; base += MT_XU * nthr) {
        float4 v[MT_XU], w[MT_XU];
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            const int t = base + j * nthr;
            v[j] = w[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < n4) {
                v[j] = __ldcg(x4 + t);
                if (aux) w[j] = __ldcg(w4 + t);
            }
        }
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            const int t = base + j * nthr;
            if (t < n4) mt_quantise4<S16, A>(a, K, xq, t, v[j], w[j], rs);
        }
    }
}

// ---- tensor-parallel exchange slots: {value bits, epoch} pairs written
// with one 8-byte store, so a reader that sees the epoch sees the value.
__device__ __forceinline__ void ll_store(void* p, float v, unsigned tag) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}
__device__ __forceinline__ uint4 ll_load2(const void* p) {   // two consecutive pairs
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
// Four consecutive values (p 16-byte aligned) once all four carry epoch ep;
// false after 2 s.
__device__ __forceinline__ bool ll_wait4(const uint2* p, unsigned ep, float4& out) {
    uint4 a = ll_load2(p), b = ll_load2(p + 2);
    if (a.y != ep || a.w != ep || b.y != ep || b.w != ep) {
        const uint64_t t0 = gtimer();
        do {
            if (gtimer() - t0 > MT_WAIT_NS) return false;
            a = ll_load2(p);
            b = ll_load2(p + 2);
        } while (a.y != ep || a.w != ep || b.y != ep || b.w != ep);
    }
    out = make_float4(__uint_as_float(a.x), __uint_as_float(a.z), __uint_as_float(b.x), __uint_as_float(b.z));
    return true;
}

// The thread's float4s of the RMSNorm weight for mt_quantise_x_rms.  The
// weight is a model constant, so the consumers load it before
// griddepcontrol.wait: otherwise its HBM reads queue behind this launch's own
// weight stream on the critical path after the wait.
template <int NC, class A>
__device__ __forceinline__ void mt_load_norm_w(const A& a, int K, int tid, float4 (&w)[MT_XU]) {
    const int n4 = K / 4, nthr = NC * 32;
    const float4* w4 = reinterpret_cast<const float4*>(a.nw);
#pragma unroll
    for (int j = 0; j < MT_XU; j++) {
        const int t = tid + j * nthr;
        w[j] = t < n4 ? __ldg(w4 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Tensor-parallel exchange on the way in (ex->in_call >= 0, epoch ep): this
// CTA's slice of x plus the sum over ranks, in rank order, of this rank's
// receive slots goes to ex->h_out; one release flag per CTA publishes it, and
// once every CTA's flag carries ep the whole new hidden state is in h_out.
// Each slot is read by one CTA only.  Returns the array to read x from.
template <int NC>
__device__ __forceinline__ const float4* mt_exchange_in(const float4* x4, int n4, int tid, const MvTp* ex,
                                                        unsigned ep) {
    const int world = ex->world;
    const uint2* slots = static_cast<const uint2*>(ex->peers[ex->rank]) + (size_t)(ep & 1) * world * ex->H;
    const int lo = (int)((long long)blockIdx.x * n4 / gridDim.x), hi = (int)((long long)(blockIdx.x + 1) * n4 / gridDim.x);
    bool ok = true;
    for (int t = lo + tid; t < hi; t += NC * 32) {
        float4 v = __ldcg(x4 + t);
        for (int q = 0; q < world; q++) {
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok && !ll_wait4(slots + (size_t)q * ex->H + 4 * t, ep, f)) {
                ok = false;
                atomicExch(ex->err, (unsigned)(-GB_ETIMEOUT));
            }
            v = make_float4(v.x + f.x, v.y + f.y, v.z + f.z, v.w + f.w);
        }
        __stcg(reinterpret_cast<float4*>(ex->h_out) + t, v);
    }
    mt_consumer_sync<NC>();   // the CTA's slice is written
    if (tid == 0)   // one release for the slice: fence at GPU scope, then the flag
        asm volatile("fence.acq_rel.gpu;\n\tst.relaxed.gpu.global.u32 [%0], %1;" ::"l"(ex->ready + blockIdx.x), "r"(ep)
                     : "memory");
    if (tid < 32) {   // wait (bounded) until every CTA's flag has reached ep
        for (int c = tid; c < (int)gridDim.x; c += 32) {
            const unsigned* f = ex->ready + c;
            if ((int)(ld_acquire(f) - ep) < 0) {
                const uint64_t t0 = gtimer();
                while ((int)(ld_acquire(f) - ep) < 0)
                    if (gtimer() - t0 > MT_WAIT_NS) {
                        atomicExch(ex->err, (unsigned)(-GB_ETIMEOUT));
                        break;
                    }
            }
        }
    }
    mt_consumer_sync<NC>();   // warp 0's acquires order every thread's reads below
    return reinterpret_cast<const float4*>(ex->h_out);
}

// RMSNorm and quantisation in one pass (K / 4 <= MT_XU * NC * 32): every
// float4 of x and of the weight is loaded once, the sum of squares reduced
// (same order as mt_rms_scale, so the same scale), then the registers are
// quantised.  One round trip to L2 instead of two.  scratch: NC floats.
// With an exchange ex (ex->in_call >= 0, epoch ep), x is the hidden state
// after the exchange (mt_exchange_in).
template <bool S16, int NC, class A>
__device__ __forceinline__ void mt_quantise_x_rms(const A& a, int K, uint8_t* xq, int tid, float* scratch,
                                                  const float4 (&w)[MT_XU], const MvTp* ex = nullptr,
                                                  unsigned ep = 0) {
    const int n4 = K / 4, nthr = NC * 32;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4 v[MT_XU];
    if (ex && !ex->ready) {
        // direct form (few ranks): every CTA adds all ranks' slots to x
        // itself, in rank order, and writes its slice of the sum to h_out
        const int world = ex->world;
        const uint2* slots = static_cast<const uint2*>(ex->peers[ex->rank]) + (size_t)(ep & 1) * world * ex->H;
        const int lo = (int)((long long)blockIdx.x * n4 / gridDim.x), hi = (int)((long long)(blockIdx.x + 1) * n4 / gridDim.x);
        bool ok = true;
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            const int t = tid + j * nthr;
            v[j] = t < n4 ? __ldcg(x4 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (t >= n4) continue;
            for (int q = 0; q < world; q++) {
                float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ok && !ll_wait4(slots + (size_t)q * ex->H + 4 * t, ep, f)) {
                    ok = false;
                    atomicExch(ex->err, (unsigned)(-GB_ETIMEOUT));
                }
                v[j] = make_float4(v[j].x + f.x, v[j].y + f.y, v[j].z + f.z, v[j].w + f.w);
            }
            if (t >= lo && t < hi) reinterpret_cast<float4*>(ex->h_out)[t] = v[j];
        }
    } else {
        if (ex) x4 = mt_exchange_in<NC>(x4, n4, tid, ex, ep);   // slice form
#pragma unroll
        for (int j = 0; j < MT_XU; j++) {
            const int t = tid + j * nthr;
            v[j] = t < n4 ? __ldcg(x4 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MT_XU; j++) {
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) scratch[tid >> 5] = ss;
    mt_consumer_sync<NC>();
    float tot = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < NC; w2++) tot += scratch[w2];
    const float rs = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
#pragma unroll
    for (int j = 0; j < MT_XU; j++) {
        const int t = tid + j * nthr;
        if (t < n4) mt_quantise4<S16, A>(a, K, xq, t, v[j], w[j], rs);
    }
}

// Per-lane constants of the tensor-core fragment map (g = lane / 4 is the
// row within an 8-row half tile and the B column; c = lane % 4 the column
// group).  Only lanes with c == g / 2 carry nonzero B fragments; the others
// read a zero line, with a zero stride, so no lane branches.  The first MMA of
// a k-step takes limbs x0, x1 (columns 2c, 2c + 1), a second one the third
// limb x2 (column 2c; column 2c + 1 zero) with the same A fragment.
struct MtLane {
    int gq, c;
    const uint8_t* xlb;   // B fragment base (limb gq & 1 of column group c)
    int xstr;             // bytes per 256-column block (0 for zero lanes)
    const uint8_t* x2b;   // B fragment base of the third limb (column 2c of the second MMA)
    int x2str;            // its bytes per block (0: a zero column)
};

// ---------------------------------------------------------------- Q4_K stage
// Box {18 x u64, 32 rows, 16 blocks}: shared layout [block][row][144 B].  Warp
// w takes block w of the stage, both 16-row tiles.
// Stage layouts: RPV == 0 is block-major [block][row][144 B] (3-D boxes of
// 144-byte rows); RPV > 0 is row-major [row][RPV B] (2-D boxes whose rows
// are KC blocks plus 16 bytes: RPV = 144 KC + 16, a pitch of 4 banks mod 32,
// so the 8 rows a quarter-warp reads fall in distinct banks, and a box
// moves KC blocks of a row per TMA request instead of one).
template <int IGV, int KCV = 16, int RPV = 0>
struct MtQ4KT {
    static constexpr int NC = 16;        // consumer warps
    static constexpr int KC = KCV;       // blocks per stage
    static constexpr int RP = RPV;
    static_assert(RP == 0 || RP == KC * GB_Q4K_BYTES + 16, "row pitch: KC blocks + 16 bytes");
    // 16-block stages: warp w takes block w, both 16-row tiles; 8-block
    // stages: warp w takes tile w / 8 of block w % 8
    static constexpr int TPW = 2 * KC / NC;
    static_assert(TPW == 1 || TPW == 2, "one or two tiles per warp");
    static constexpr int STG = RP ? MT_GR * RP : KC * MT_GR * GB_Q4K_BYTES;
    static constexpr bool S16 = false;
    static constexpr int XB_LANE = 64;   // B fragment offset per column group
    static constexpr int IG = IGV;       // blocks per split item
    static constexpr int SI = KC / IG;   // items per full stage
    static constexpr int ITEM = STG / SI;
    static constexpr int ZUNIT = 1;      // blocks per tensor-map z unit
    static constexpr int BOXZ = IG;      // box depth: one box per item
    // blocks [b0, bend) of the group land at stage blocks 0 .. bend - b0 - 1
    __device__ static __forceinline__ void consume(const uint8_t* stg, int b0, int bend, int warp, const MtLane& L,
                                                   const uint8_t* xq, int K, float acc_a[2], float acc_b[2]) {
        const int gq = L.gq, c = L.c;
        const int bl = TPW == 2 ? warp : (warp % KC);
        const int mfirst = TPW == 2 ? 0 : warp / KC;
        const int b = b0 + bl;
        if (b >= bend) return;
        const float4* xfb = reinterpret_cast<const float4*>(xq + 3 * K) + c;
        const int sh8 = (c & 1) << 4;
        const uint32_t MW = c >= 2 ? 0x0F0Fu : 0u, MY = c >= 2 ? 0x3030u : 0x3F3Fu, SY = c >= 2 ? 2u : 0u;
        const uint4* xb = reinterpret_cast<const uint4*>(L.xlb + b * L.xstr);
        const uint4 bl0 = xb[0], bl1 = xb[1], bh0 = xb[2], bh1 = xb[3];
        const uint8_t* x2 = L.x2b + b * L.x2str;   // third limb: lo sub-block at 8u, hi at 32 + 8u
        const float4 xf = xfb[b * 4];
        const float xlo = xf.x * 0.00390625f, xhi = xf.y * (0.00390625f * 0.0625f);
#pragma unroll
        for (int mi = 0; mi < TPW; mi++) {   // the warp's 16-row tiles
            const int m = mfirst + mi;
            const uint8_t* ra = RP ? stg + (m * 16 + gq) * RP + bl * GB_Q4K_BYTES
                                   : stg + bl * (MT_GR * GB_Q4K_BYTES) + (m * 16 + gq) * GB_Q4K_BYTES;
            const uint8_t* rb = ra + 8 * (RP ? RP : GB_Q4K_BYTES);
            const uint4 ha = *reinterpret_cast<const uint4*>(ra);
            const uint4 hb = *reinterpret_cast<const uint4*>(rb);
            const uint4 qa0 = *reinterpret_cast<const uint4*>(ra + 16 + 32 * c);
            const uint4 qa1 = *reinterpret_cast<const uint4*>(ra + 32 + 32 * c);
            const uint4 qb0 = *reinterpret_cast<const uint4*>(rb + 16 + 32 * c);
            const uint4 qb1 = *reinterpret_cast<const uint4*>(rb + 32 + 32 * c);
            int4 cl = make_int4(0, 0, 0, 0), chh = make_int4(0, 0, 0, 0);
            int4 cl2 = make_int4(0, 0, 0, 0), ch2 = make_int4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint4& qa = (u >> 1) ? qa1 : qa0;
                const uint4& qb = (u >> 1) ? qb1 : qb0;
                const uint32_t wa0 = (u & 1) ? qa.z : qa.x, wa1 = (u & 1) ? qa.w : qa.y;
                const uint32_t wb0 = (u & 1) ? qb.z : qb.x, wb1 = (u & 1) ? qb.w : qb.y;
                const uint4& blx = (u >> 1) ? bl1 : bl0;
                const uint4& bhx = (u >> 1) ? bh1 : bh0;
                const uint32_t l0 = (u & 1) ? blx.z : blx.x, l1 = (u & 1) ? blx.w : blx.y;
                const uint32_t h0 = (u & 1) ? bhx.z : bhx.x, h1 = (u & 1) ? bhx.w : bhx.y;
                const uint2 tl = *reinterpret_cast<const uint2*>(x2 + 8 * u);
                const uint2 th = *reinterpret_cast<const uint2*>(x2 + 32 + 8 * u);
                const uint32_t m0 = tl.x, m1 = tl.y, n0 = th.x, n1 = th.y;
                const uint32_t la0 = wa0 & 0x0F0F0F0Fu, lb0 = wb0 & 0x0F0F0F0Fu, la1 = wa1 & 0x0F0F0F0Fu,
                               lb1 = wb1 & 0x0F0F0F0Fu;
                const uint32_t ha0 = wa0 & 0xF0F0F0F0u, hb0 = wb0 & 0xF0F0F0F0u, ha1 = wa1 & 0xF0F0F0F0u,
                               hb1 = wb1 & 0xF0F0F0F0u;
                mma_u8s8(cl, la0, lb0, la1, lb1, l0, l1);
                mma_u8s8(chh, ha0, hb0, ha1, hb1, h0, h1);
                mma_u8s8(cl2, la0, lb0, la1, lb1, m0, m1);
                mma_u8s8(ch2, ha0, hb0, ha1, hb1, n0, n1);
            }
            // sub-blocks 2c (low nibbles) and 2c + 1 (high nibbles) of rows a, b
            float pab[2];
#pragma unroll
            for (int w = 0; w < 2; w++) {
                const uint4 h = w ? hb : ha;
                const uint32_t y = h.y >> sh8, z = h.z >> sh8, ww = h.w >> sh8;
                const uint32_t sc = (ww & MW) | ((y >> SY) & MY);
                const uint32_t mn = ((ww >> 4) & MW) | ((z >> SY) & MY);
                const float sc_lo = (float)(sc & 0xFFu), sc_hi = (float)((sc >> 8) & 0xFFu);
                const float m_lo = (float)(mn & 0xFFu), m_hi = (float)((mn >> 8) & 0xFFu);
                const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const int dl = (w ? cl.z : cl.x) * 256 + (w ? cl.w : cl.y);
                const int dh = (w ? chh.z : chh.x) * 256 + (w ? chh.w : chh.y);
                const float fl = fmaf((float)(w ? cl2.z : cl2.x), 0.00390625f, (float)dl);
                const float fh = fmaf((float)(w ? ch2.z : ch2.x), 0.00390625f, (float)dh);
                const float tt = (sc_lo * xlo) * fl + (sc_hi * xhi) * fh;
                const float mm = m_lo * xf.z + m_hi * xf.w;
                pab[w] = fmaf(dm.x, tt, -dm.y * mm);
            }
            if (m == 0) {
                acc_a[0] += pab[0];
                acc_b[0] += pab[1];
            } else {
                acc_a[1] += pab[0];
                acc_b[1] += pab[1];
            }
        }
    }
};
// 16-block items: a stage is one box and a 32-row group of a 4096-column
// matrix is one item, so such launches split by whole groups
using MtQ4K = MtQ4KT<16>;

// ---------------------------------------------------------------- Q6_K stage
// Box {210 x u64 = 8 blocks, 32 rows, 1 chunk}: shared layout [row][1680 B];
// warp w takes block w of every row, so its blocks start at 210 w within a
// row and every field of the block sits at the same offset mod 8, MIS =
// (2 w) mod 8.  Loads are specialised on MIS: 64-bit when aligned, two words
// at 4, three words and two byte permutes at 2 or 6.
template <int MIS>
__device__ __forceinline__ uint2 lds8_mis(const uint8_t* p) {
    if constexpr (MIS == 0) {
        return *reinterpret_cast<const uint2*>(p);
    } else if constexpr (MIS == 4) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
        return make_uint2(w[0], w[1]);
    } else {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(p - 2);
        const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
        return make_uint2(__byte_perm(w0, w1, 0x5432), __byte_perm(w1, w2, 0x5432));
    }
}
// 6-bit codes of weights 128 n + 32 G + [8c, 8c + 8) from the ql / qh words
// (low / high word of the lane's 8 bytes): low nibble for G < 2, high for
// G >= 2; ql from byte 8c (G even) or 32 + 8c (G odd); qh bits 2G..2G+1.
// Byte of w chosen by the prmt selector sel, sign-extended (prmt selector
// nibbles with bit 3 set replicate the sign of the chosen byte).
__device__ __forceinline__ int prmt_sext(uint32_t w, int sel) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return r;
}
template <int G>
__device__ __forceinline__ uint32_t q6_code(uint32_t lw, uint32_t hw) {
    const uint32_t nib = (G >> 1) ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
    const uint32_t hi = G == 0 ? (hw << 4) : G == 1 ? (hw << 2) : G == 2 ? hw : (hw >> 2);
    return nib | (hi & 0x30303030u);
}
struct MtQ6K {
    static constexpr int NC = 16;        // consumer warps: block w % 8, 16-row tile w / 8
    static constexpr int KC = 8;
    static constexpr int RB = 8 * GB_Q6K_BYTES;   // 1680 bytes per row per stage
    static constexpr int STG = MT_GR * RB;
    static constexpr bool S16 = true;
    static constexpr int XB_LANE = 8;
    static constexpr int IG = 8;         // blocks per split item: one 16-byte aligned 1680-byte row run
    static constexpr int SI = 1;         // items per stage
    static constexpr int ITEM = STG;
    static constexpr int ZUNIT = 8;      // blocks per tensor-map z unit
    static constexpr int BOXZ = 1;
    template <int MIS>
    __device__ static __forceinline__ void tile(const uint8_t* blk_a, int c, const uint8_t* xb, const uint8_t* x2b,
                                                const float* xf,
                                                const float4 s16lo, const float4 s16hi, float fc, int selsc0,
                                                int selsc1, float& acc_a, float& acc_b) {
        const uint8_t* blk_b = blk_a + 8 * RB;
        const uint8_t* ra = blk_a + 8 * c;   // the lane's 8 bytes of each 32-byte ql / qh run
        const uint8_t* rb = blk_b + 8 * c;
        float ba = 0.f, bb = 0.f;   // block sums before the super-scale d
        // int8 scales of rows a and b, 16 bytes at 192
        uint32_t sa[4], sb[4];
        {
            const uint2 a0 = lds8_mis<MIS>(blk_a + 192), a1 = lds8_mis<MIS>(blk_a + 200);
            const uint2 b0 = lds8_mis<MIS>(blk_b + 192), b1 = lds8_mis<MIS>(blk_b + 200);
            sa[0] = a0.x; sa[1] = a0.y; sa[2] = a1.x; sa[3] = a1.y;
            sb[0] = b0.x; sb[1] = b0.y; sb[2] = b1.x; sb[3] = b1.y;
        }
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const uint2 qa0 = lds8_mis<MIS>(ra + 64 * n), qa1 = lds8_mis<MIS>(ra + 64 * n + 32);
            const uint2 qb0 = lds8_mis<MIS>(rb + 64 * n), qb1 = lds8_mis<MIS>(rb + 64 * n + 32);
            const uint2 ha = lds8_mis<MIS>(ra + 128 + 32 * n), hb = lds8_mis<MIS>(rb + 128 + 32 * n);
            const float4 xs = *reinterpret_cast<const float4*>(xf + 8 * n);       // sub-blocks 4n, 4n+1
            const float4 xs2 = *reinterpret_cast<const float4*>(xf + 8 * n + 4);  // sub-blocks 4n+2, 4n+3
#pragma unroll
            for (int G = 0; G < 4; G++) {
                const uint2& la = (G & 1) ? qa1 : qa0;
                const uint2& lb = (G & 1) ? qb1 : qb0;
                uint32_t A0, A1, A2, A3;
                switch (G) {
                    case 0: A0 = q6_code<0>(la.x, ha.x); A1 = q6_code<0>(lb.x, hb.x); A2 = q6_code<0>(la.y, ha.y); A3 = q6_code<0>(lb.y, hb.y); break;
                    case 1: A0 = q6_code<1>(la.x, ha.x); A1 = q6_code<1>(lb.x, hb.x); A2 = q6_code<1>(la.y, ha.y); A3 = q6_code<1>(lb.y, hb.y); break;
                    case 2: A0 = q6_code<2>(la.x, ha.x); A1 = q6_code<2>(lb.x, hb.x); A2 = q6_code<2>(la.y, ha.y); A3 = q6_code<2>(lb.y, hb.y); break;
                    default: A0 = q6_code<3>(la.x, ha.x); A1 = q6_code<3>(lb.x, hb.x); A2 = q6_code<3>(la.y, ha.y); A3 = q6_code<3>(lb.y, hb.y); break;
                }
                const uint2 bf = *reinterpret_cast<const uint2*>(xb + 128 * n + 32 * G);
                const uint2 bf2 = *reinterpret_cast<const uint2*>(x2b + 128 * n + 32 * G);
                int4 cc = make_int4(0, 0, 0, 0), cc2 = make_int4(0, 0, 0, 0);
                mma_u8s8(cc, A0, A1, A2, A3, bf.x, bf.y);
                mma_u8s8(cc2, A0, A1, A2, A3, bf2.x, bf2.y);
                const float xsg = ((G >> 1) ? ((G & 1) ? xs2.y : xs2.x) : ((G & 1) ? xs.y : xs.x)) * 0.00390625f;
                const float s16 = n ? ((G == 0) ? s16hi.x : (G == 1) ? s16hi.y : (G == 2) ? s16hi.z : s16hi.w)
                                    : ((G == 0) ? s16lo.x : (G == 1) ? s16lo.y : (G == 2) ? s16lo.z : s16lo.w);
                // scale byte 8n + 2G + (c >> 1): word 2n + (G >> 1), byte 2 (G & 1) + (c >> 1)
                const int sel = (G & 1) ? selsc1 : selsc0;
                const float sca = (float)prmt_sext(sa[2 * n + (G >> 1)], sel);
                const float scb = (float)prmt_sext(sb[2 * n + (G >> 1)], sel);
                const float ta = fmaf(xsg, fmaf((float)cc2.x, 0.00390625f, (float)(cc.x * 256 + cc.y)), fc * s16);
                const float tb = fmaf(xsg, fmaf((float)cc2.z, 0.00390625f, (float)(cc.z * 256 + cc.w)), fc * s16);
                ba = fmaf(sca, ta, ba);
                bb = fmaf(scb, tb, bb);
            }
        }
        const float da = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk_a + 208)));
        const float db = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk_b + 208)));
        acc_a = fmaf(da, ba, acc_a);
        acc_b = fmaf(db, bb, acc_b);
    }
    template <int MIS>
    __device__ static __forceinline__ void run(const uint8_t* stg, int b, int warp, const MtLane& L, const uint8_t* xq,
                                               int K, float acc_a[2], float acc_b[2]) {
        const int c = L.c;
        const uint8_t* xb = L.xlb + b * L.xstr;
        const uint8_t* x2b = L.x2b + b * L.x2str;
        const float* xf = reinterpret_cast<const float*>(xq + 3 * K) + b * 16;   // {s, s, sum, sum} x 4
        // xf holds per 64-column chunk {s lo, s hi, sum lo, sum hi}: the scale
        // of 32-column sub-block 4n + G is xf[8n + 4 (G >> 1) + (G & 1)]
        const float* f16 = reinterpret_cast<const float*>(xq + 3 * K + K / 4) + b * 16 + (c >> 1) * 8;
        const float4 s16lo = *reinterpret_cast<const float4*>(f16);
        const float4 s16hi = *reinterpret_cast<const float4*>(f16 + 4);
        const float fc = (c & 1) ? 0.f : -32.f;   // the -32 offset of the codes, once per 16 columns
        const int h = c >> 1;
        // prmt selectors extracting byte 2 (G & 1) + h sign-extended
        const int b0 = h, b1 = 2 + h;
        const int selsc0 = b0 | ((b0 | 8) << 4) | ((b0 | 8) << 8) | ((b0 | 8) << 12);
        const int selsc1 = b1 | ((b1 | 8) << 4) | ((b1 | 8) << 8) | ((b1 | 8) << 12);
        const int m = warp >> 3;
        const uint8_t* blk = stg + (m * 16 + L.gq) * RB + (warp & 7) * GB_Q6K_BYTES;
        tile<MIS>(blk, c, xb, x2b, xf, s16lo, s16hi, fc, selsc0, selsc1, acc_a[m], acc_b[m]);
    }
    __device__ static __forceinline__ void consume(const uint8_t* stg, int b0, int bend, int warp, const MtLane& L,
                                                   const uint8_t* xq, int K, float acc_a[2], float acc_b[2]) {
        const int b = b0 + (warp & 7);
        if (b >= bend) return;
        switch ((2 * warp) & 7) {
            case 0: run<0>(stg, b, warp, L, xq, K, acc_a, acc_b); break;
            case 2: run<2>(stg, b, warp, L, xq, K, acc_a, acc_b); break;
            case 4: run<4>(stg, b, warp, L, xq, K, acc_a, acc_b); break;
            default: run<6>(stg, b, warp, L, xq, K, acc_a, acc_b); break;
        }
    }
};

}  // namespace gb
