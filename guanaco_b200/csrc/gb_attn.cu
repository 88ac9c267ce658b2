// gb_attn.cu -- single-query GQA decode attention fused with RoPE and the KV
// append, split across CTAs over the context and merged with an online-softmax
// reduction.
//
// Reference semantics (T = 1): src/engine/engine.c:372-509 --
//   rope(q, k, pos)                       kernels_cpu.c:391-431
//   kv_cache_append(k, v, pos)            kv_cache.c:95-128 (slot pos % max_seq)
//   for each q head h, kv head h / (n_heads / n_kv):
//     s = (q . K[t]) * (1/sqrt(hd)),  p = softmax(s over t = 0..pos),
//     out_h = sum_t p_t V[t]
// Replaces cuda_update_kv_cache_kernel, cuda_attn_scores_kernel_gqa,
// cuda_softmax_kernel and cuda_attn_context_kernel_gqa
// (src/kernels/cuda/cuda_layer_kernels.cu:425-504).
//
// Layout: the KV cache keeps the reference's fp32 head-major layout
// [n_kv][max_seq][head_dim] per layer (kv_cache.c:90-93).
//
// Shape: grid = n_kv * grid_splits CTAs, one CTA per SM over all KV heads.
// A CTA owns one KV head and P consecutive positions (P from pos, so the
// active splits fill the grid); it serves all GROUP = n_heads / n_kv query
// heads of that KV head, so each K and V row is read from HBM exactly once.
// One producer lane streams K and V tiles of 32 positions through a ring of
// bulk copies (about 200 KB per SM in flight), starting before RoPE; the 16
// consumer warps form TW tile lanes of NHG warps (one per group of HPW query
// heads): tile t belongs to tile lane t % TW, and each warp runs its own
// online softmax, with no CTA-wide barrier per tile:
//   scores:  LPP lanes share one K row (DPL dims each, 128-bit loads), dot
//            products for the warp's HPW heads, shuffle-reduced;
//   softmax: per head, the tile's max updates the warp's running max m, and
//            the running sum l and the output are rescaled by exp(m_old - m);
//   P.V:     each lane accumulates one float4 column of every head;
//   merge:   the warps' (m, l, o) combine in shared memory, each CTA
//            publishes its (m, l, o[hd]) per head with one release (ticket),
//            and the last CTA of the KV head combines the splits in split
//            order, resets the ticket and, when asked, also writes the output
//            quantised for the next matvec.
// pos comes from device memory so the launch can live inside a CUDA graph;
// a pos outside [0, max_seq) sets the error word and touches nothing.
#include "gb_common.cuh"
#include "gb_internal.h"
#include "gb_mt.cuh"

#include <mutex>

namespace gb {

constexpr int ATTN_CWARPS = 16;                       // consumer warps
constexpr int ATTN_THREADS = (ATTN_CWARPS + 1) * 32;   // + the producer warp
constexpr int ATTN_SMEM_MAX = 227 * 1024;
// A split's partial per query head: {m, l, 2 pad, o[head_dim]} (o 16-byte
// aligned for the float4 merge).
__host__ __device__ constexpr int attn_part_stride(int hd) { return hd + 4; }
// Fewest positions a split takes (two 32-position tiles): with few KV heads
// per GPU (tensor parallelism) the context is not cut into more splits than
// the merge can combine quickly.
constexpr int ATTN_MIN_SPLIT_POS = 64;

// Splits per KV head: one CTA per SM over all heads (every split then has
// its whole share of K/V requested nearly at once), at least one 32-position
// tile per split.
// GB_ATTN_SPLITS=n in the environment caps the splits per KV head.
static int attn_split_cap() {
    static const int v = [] {
        const char* e = getenv("GB_ATTN_SPLITS");
        return e ? atoi(e) : 0;
    }();
    return v;
}

int attn_grid_splits(int n_kv, int max_seq) {
    int s = sm_count() / n_kv;
    if (attn_split_cap() > 0 && s > attn_split_cap()) s = attn_split_cap();
    if (s < 1) s = 1;
    const int tiles = (max_seq + 31) / 32;
    return s < tiles ? s : tiles;
}

template <int HD, int GROUP>
struct AttnCfg {
    // a warp serves HPW query heads of one tile: NHG head groups, so TW warps
    // (tile lanes) work on different tiles at the same time
    static constexpr int HPW = GROUP < 2 ? GROUP : 2;
    static constexpr int NHG = GROUP / HPW;
    static constexpr int TW = ATTN_CWARPS / NHG;
    static constexpr int DPL = 16;                    // K dims per lane (scores)
    static constexpr int LPP = HD / DPL;              // lanes per K row
    static constexpr int PPW = 32 / LPP;              // K rows per warp step
    static constexpr int TP = 32;                     // positions per K / V tile
    static constexpr int TILE = TP * HD;              // floats per tile
    static constexpr int CH = HD / 4;                 // float4 columns of a V row
    static constexpr int RPL = 32 / CH;               // rows a warp's P.V step covers
    // shared: q[GROUP][HD] | k_new[HD] | v_new[HD] | per-warp p[TP][2] |
    // spare [8] | issued-item count [4] | ring[R][TILE] | full[R], empty[R]
    static constexpr int HEAD_FLOATS = GROUP * HD + 2 * HD + ATTN_CWARPS * TP * 2 + 8 + 4;
    static constexpr size_t RING_OFF = ((size_t)HEAD_FLOATS * sizeof(float) + 127) / 128 * 128;
    static constexpr int R0 = (int)((ATTN_SMEM_MAX - RING_OFF - 512) / (TILE * sizeof(float)));
    static constexpr int R = R0 < 24 ? R0 : 24;       // items (K or V tiles) in flight per CTA
    static constexpr size_t BAR_OFF = RING_OFF + (size_t)R * TILE * sizeof(float);
    static constexpr size_t SMEM = BAR_OFF + 2 * R * sizeof(unsigned long long);
    // the warps' (m, l, o) merge reuses the ring
    static_assert(TW * GROUP * (HD + 4) <= R * TILE, "merge buffers");
};

// ---- bulk-copy ring primitives (shared-memory addresses)
__device__ __forceinline__ uint32_t a_sptr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void a_bar_init(uint32_t b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void a_bar_expect(uint32_t b, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(tx) : "memory");
}
__device__ __forceinline__ bool a_bar_test(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t a_gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait (2 s); false on timeout (the caller records GB_ETIMEOUT).
__device__ __noinline__ bool a_bar_wait_slow(uint32_t b, uint32_t parity) {
    const uint64_t t0 = a_gtimer();
    while (!a_bar_test(b, parity))
        if (a_gtimer() - t0 > 2000000000ull) return false;
    return true;
}
__device__ __forceinline__ bool a_bar_wait(uint32_t b, uint32_t parity) {
    return a_bar_test(b, parity) || a_bar_wait_slow(b, parity);
}
__device__ __forceinline__ void a_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void a_bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}

template <int HD, int GROUP>
__global__ void __launch_bounds__(ATTN_THREADS, 1)
k_attn_decode(const float* __restrict__ q, const float* __restrict__ knew, const float* __restrict__ vnew,
              float* __restrict__ kc, float* __restrict__ vc, const float* __restrict__ rope_cs,
              const int* __restrict__ d_pos, int n_kv, int max_seq, int grid_splits,
              float* __restrict__ out, float* __restrict__ part, unsigned* __restrict__ tickets,
              unsigned* __restrict__ err, uint8_t* __restrict__ xq_out) {
    using C = AttnCfg<HD, GROUP>;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // wo may start its weight prefetch
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                       // [GROUP][HD] rotated q
    float* kn = qs + GROUP * HD;          // [HD] rotated new k
    float* vn = kn + HD;                  // [HD] new v
    float* pw_all = vn + HD;              // [CWARPS][TP][2] each warp's scores, then probabilities
    float* spare = pw_all + ATTN_CWARPS * C::TP * 2;   // [8] unused
    // items the producer has issued: a consumer waits for its item to be
    // issued before it waits on the slot's barrier (a slot's barrier only
    // tells one generation from the next, and warps wait out of item order)
    volatile int* issued = reinterpret_cast<volatile int*>(spare + 8);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvh = blockIdx.x / grid_splits, split = blockIdx.x % grid_splits;
    const int pos = *d_pos;
    if (pos < 0 || pos >= max_seq) {
        if (blockIdx.x == 0 && tid == 0) atomicExch(err, (unsigned)(-GB_EPOS));
        return;
    }
    const int seq = pos + 1;
    // positions per split: any count (a copy is whole 512-byte rows), so every
    // split of the grid gets work
    const int P = max((seq + grid_splits - 1) / grid_splits, ATTN_MIN_SPLIT_POS);
    const int nsplit = (seq + P - 1) / P;
    if (split >= nsplit) return;
    const int s0 = split * P, n = min(seq, s0 + P) - s0;
    const bool owner = pos >= s0 && pos < s0 + n;   // this split holds the new row
    const size_t head_base = (size_t)kvh * max_seq * HD;
    const int T = (n + C::TP - 1) / C::TP;

    unsigned char* smb = reinterpret_cast<unsigned char*>(sm);
    float* ring = reinterpret_cast<float*>(smb + C::RING_OFF);
    const uint32_t full = a_sptr(smb + C::BAR_OFF), empty = full + 8 * C::R;

    // ---- items: 2t = K tile t, 2t + 1 = V tile t, in slot item % R.  Tile t
    // belongs to the NHG consumer warps of tile lane t % TW (one per group of
    // HPW query heads), which release both of its slots.
    // The row of the new position is read from kn / vn, never from a tile
    // (the copy may precede the append).  The producer starts the stream at
    // once and only arrives on barrier 2, so RoPE runs on the consumer warps
    // while the first tiles are in flight.
    if (warp == ATTN_CWARPS) {   // ---- producer
        if (lane == 0) {
            for (int r = 0; r < C::R; r++) {
                a_bar_init(full + 8 * r, 1);
                a_bar_init(empty + 8 * r, C::NHG);   // the warps that own the tile release it
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            *issued = 0;
            __threadfence_block();
        }
        __syncwarp();
        asm volatile("bar.arrive 2, %0;" ::"n"(ATTN_THREADS) : "memory");   // barriers and count ready
        if (lane == 0) {
            bool ok = true;
            int it = 0;
            for (; it < 2 * T; it++) {
                const int sl = it % C::R;
                if (it >= C::R && !a_bar_wait(empty + 8 * sl, ((it / C::R) - 1) & 1)) {
                    ok = false;
                    atomicExch(err, (unsigned)(-GB_ETIMEOUT));
                    break;
                }
                const int t = it >> 1;
                const int rows = min(C::TP, n - t * C::TP);
                const float* src = ((it & 1) ? vc : kc) + head_base + (size_t)(s0 + t * C::TP) * HD;
                a_bar_expect(full + 8 * sl, rows * HD * 4);
                a_bulk_g2s(a_sptr(ring + sl * C::TILE), src, rows * HD * 4, full + 8 * sl);
                __threadfence_block();
                *issued = it + 1;
            }
            // do not retire while a copy may still be landing in the ring
            for (int j = it > C::R ? it - C::R : 0; ok && j < it; j++)
                if (!a_bar_wait(empty + 8 * (j % C::R), (j / C::R) & 1)) {
                    ok = false;
                    atomicExch(err, (unsigned)(-GB_ETIMEOUT));
                }
        }
        return;
    }

    // q, k, v come from the previous kernel: with programmatic dependent
    // launch the producer above already streams the cached K / V (written by
    // earlier steps), the consumers wait here for the projections
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // ---- RoPE on the consumer warps (reference rounding: a*c - b*s,
    // a*s + b*c, no contraction)
    constexpr int CT = ATTN_CWARPS * 32;   // consumer threads
    const float* cs = rope_cs + (size_t)pos * HD;
    for (int e = tid; e < (GROUP + 1) * (HD / 2); e += CT) {
        const int h = e / (HD / 2), i = e % (HD / 2);
        const float* src = h < GROUP ? q + (size_t)(kvh * GROUP + h) * HD : knew + (size_t)kvh * HD;
        float* dst = h < GROUP ? qs + h * HD : kn;
        const float a = src[2 * i], b = src[2 * i + 1], c = cs[2 * i], s = cs[2 * i + 1];
        dst[2 * i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        dst[2 * i + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    for (int i = tid; i < HD; i += CT) vn[i] = vnew[(size_t)kvh * HD + i];
    asm volatile("bar.sync 2, %0;" ::"n"(ATTN_THREADS) : "memory");   // with the producer's arrival
    if (owner) {   // KV append at slot pos (the ring index pos % max_seq == pos here)
        for (int i = tid; i < HD; i += CT) {
            kc[head_base + (size_t)pos * HD + i] = kn[i];
            vc[head_base + (size_t)pos * HD + i] = vn[i];
        }
    }

    // ---- consumer warps: each runs its own online softmax over its tiles
    // for its HPW query heads hg * HPW ..
    const int hg = warp / C::TW, tl = warp % C::TW;
    const float scale = 1.0f / sqrtf((float)HD);
    const int lp = lane % C::LPP, pw = lane / C::LPP;
    float qr[C::HPW][C::DPL];
#pragma unroll
    for (int j = 0; j < C::HPW; j++)
#pragma unroll
        for (int i = 0; i < C::DPL / 4; i++) {
            const float4 v = *reinterpret_cast<const float4*>(qs + (hg * C::HPW + j) * HD + i * C::LPP * 4 + lp * 4);
            qr[j][4 * i] = v.x; qr[j][4 * i + 1] = v.y; qr[j][4 * i + 2] = v.z; qr[j][4 * i + 3] = v.w;
        }
    float* pw2 = pw_all + warp * C::TP * 2;   // this warp's [TP][2]
    const int ch = lane % C::CH, rl = lane / C::CH;
    float m[C::HPW], l[C::HPW];
    float4 acc[C::HPW];
#pragma unroll
    for (int j = 0; j < C::HPW; j++) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    bool ok = true;
    auto wait_item = [&](int it) {
        bool got = true;
        if (*issued <= it) {   // bounded (2 s), like every wait here
            const uint64_t t0 = a_gtimer();
            while (*issued <= it)
                if (a_gtimer() - t0 > 2000000000ull) { got = false; break; }
        }
        if (got) got = a_bar_wait(full + 8 * (it % C::R), (it / C::R) & 1);
        if (!got && ok) {
            ok = false;
            atomicExch(err, (unsigned)(-GB_ETIMEOUT));
        }
    };
    for (int t = tl; t < T; t += C::TW) {
        const int nt = min(C::TP, n - t * C::TP);
        const int kit = 2 * t, vit = 2 * t + 1;
        // ---- scores of K tile t: LPP lanes per row, dot products for HPW heads
        wait_item(kit);
        {
            const float* tile = ring + (kit % C::R) * C::TILE;
#pragma unroll 2
            for (int r0 = 0; r0 < nt; r0 += C::PPW) {
                const int r = r0 + pw;
                const int rr = r < nt ? r : 0;
                const float* krow = (s0 + t * C::TP + rr == pos) ? kn : tile + rr * HD;
                float4 kr[C::DPL / 4];
#pragma unroll
                for (int i = 0; i < C::DPL / 4; i++) kr[i] = *reinterpret_cast<const float4*>(krow + i * C::LPP * 4 + lp * 4);
                float dots[C::HPW];
#pragma unroll
                for (int j = 0; j < C::HPW; j++) {
                    float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < C::DPL / 4; i++) {
                        acc2 = ffma2(make_float2(qr[j][4 * i], qr[j][4 * i + 1]), make_float2(kr[i].x, kr[i].y), acc2);
                        acc2 = ffma2(make_float2(qr[j][4 * i + 2], qr[j][4 * i + 3]), make_float2(kr[i].z, kr[i].w), acc2);
                    }
                    float d = acc2.x + acc2.y;
#pragma unroll
                    for (int o = C::LPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    dots[j] = d;
                }
                if (r < nt && lp < C::HPW) pw2[r * 2 + lp] = __fmul_rn(lp ? dots[C::HPW - 1] : dots[0], scale);
            }
        }
        __syncwarp();
        if (lane == 0) a_bar_arrive(empty + 8 * (kit % C::R));   // this warp is done with the K slot
        // ---- online softmax over the tile: lane r holds row r
        float alpha[C::HPW];
#pragma unroll
        for (int j = 0; j < C::HPW; j++) {
            const float v = lane < nt ? pw2[lane * 2 + j] : -INFINITY;
            const float mn = fmaxf(m[j], warp_max(v));
            const float p = lane < nt ? expf(v - mn) : 0.f;
            alpha[j] = expf(m[j] - mn);   // 0 on the warp's first tile (m = -inf)
            l[j] = fmaf(l[j], alpha[j], warp_sum(p));
            m[j] = mn;
            pw2[lane * 2 + j] = p;
        }
        __syncwarp();
        // ---- o_h = o_h * alpha_h + sum_r p_h[r] V[r]
        wait_item(vit);
        {
            const float* vt = ring + (vit % C::R) * C::TILE;
#pragma unroll
            for (int j = 0; j < C::HPW; j++)
                acc[j] = make_float4(acc[j].x * alpha[j], acc[j].y * alpha[j], acc[j].z * alpha[j], acc[j].w * alpha[j]);
#pragma unroll 4
            for (int r = rl; r < nt; r += C::RPL) {
                const float4 vv = (s0 + t * C::TP + r == pos) ? *reinterpret_cast<const float4*>(vn + ch * 4)
                                                              : *reinterpret_cast<const float4*>(vt + r * HD + ch * 4);
                const float2 pp = *reinterpret_cast<const float2*>(pw2 + r * 2);
#pragma unroll
                for (int j = 0; j < C::HPW; j++) {
                    const float pj = j ? pp.y : pp.x;
                    float2 lo = ffma2(make_float2(pj, pj), make_float2(vv.x, vv.y), make_float2(acc[j].x, acc[j].y));
                    float2 hi = ffma2(make_float2(pj, pj), make_float2(vv.z, vv.w), make_float2(acc[j].z, acc[j].w));
                    acc[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                }
            }
        }
        __syncwarp();
        if (lane == 0) a_bar_arrive(empty + 8 * (vit % C::R));   // this warp is done with the V slot
    }
    // lanes that covered other rows of the same columns (head_dim < 128)
#pragma unroll
    for (int o = C::CH; o < 32; o <<= 1)
#pragma unroll
        for (int j = 0; j < C::HPW; j++) {
            acc[j].x += __shfl_xor_sync(0xffffffffu, acc[j].x, o);
            acc[j].y += __shfl_xor_sync(0xffffffffu, acc[j].y, o);
            acc[j].z += __shfl_xor_sync(0xffffffffu, acc[j].z, o);
            acc[j].w += __shfl_xor_sync(0xffffffffu, acc[j].w, o);
        }

    // ---- merge the warps' (m, l, o) in the ring (every tile is consumed)
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(ATTN_CWARPS * 32) : "memory");
    constexpr int WS = HD + 4;   // m, l, 2 pad, o[HD]: o stays 16-byte aligned
    float* wst = ring;           // [TW][GROUP][WS]
#pragma unroll
    for (int j = 0; j < C::HPW; j++) {
        float* w = wst + (tl * GROUP + hg * C::HPW + j) * WS;
        if (lane == 0) { w[0] = m[j]; w[1] = l[j]; }
        if (lane < C::CH) *reinterpret_cast<float4*>(w + 4 + ch * 4) = acc[j];
    }
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(ATTN_CWARPS * 32) : "memory");
    const int ctid = tid;   // 0 .. CT - 1
    const bool single = nsplit == 1;
    constexpr int PS = attn_part_stride(HD);
    float* my = part + ((size_t)kvh * grid_splits + split) * GROUP * PS;
    for (int e = ctid; e < GROUP * HD; e += ATTN_CWARPS * 32) {
        const int h = e / HD, d = e % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::TW; w++) M = fmaxf(M, wst[(w * GROUP + h) * WS]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < C::TW; w++) {
            const float* ws = wst + (w * GROUP + h) * WS;
            const float a = ws[0] == -INFINITY ? 0.f : expf(ws[0] - M);   // warps without tiles
            L = fmaf(ws[1], a, L);
            O = fmaf(ws[4 + d], a, O);
        }
        if (single) {
            out[(size_t)(kvh * GROUP + h) * HD + d] = O / L;
            // a warp holds one 32-column group: e >> 5 is warp-uniform
            if (xq_out) mt_quantise32(xq_out, n_kv * GROUP * HD, (kvh * GROUP * HD + e) >> 5, lane, O / L);
        } else {
            my[h * PS + 4 + d] = O;
            if (d == 0) { my[h * PS] = M; my[h * PS + 1] = L; }
        }
    }
    if (single) return;

    // ---- merge in the last CTA of this KV head.  One release per CTA
    // publishes its partials: after the CTA barrier thread 0 fences at GPU
    // scope and takes a ticket with an acquire-release atomic, so the last
    // arrival's thread 0 acquires every split's partials, and the barrier
    // after it orders the whole CTA's reads behind that acquire.
    __shared__ unsigned last;
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(ATTN_CWARPS * 32) : "memory");
    if (ctid == 0) {
        unsigned prev;
        asm volatile("fence.acq_rel.gpu;\n\tatom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(tickets + kvh)
                     : "memory");
        last = prev == (unsigned)(nsplit - 1);
    }
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(ATTN_CWARPS * 32) : "memory");
    if (!last) return;
    // Every output is a weighted sum over the splits.  The CTA's threads
    // split the work both ways: NV threads each own a float4 of the output
    // (head h, dims d4 .. d4 + 3), and NQ such groups take the splits
    // q, q + NQ, ... with a running maximum (loads of MC splits in flight);
    // the NQ partial (m, l, o) are then combined in q order (deterministic).
    constexpr int NV = GROUP * HD / 4;            // float4 outputs
    constexpr int NQ = CT / NV >= 1 ? CT / NV : 1;
    static_assert(CT % NV == 0, "merge thread map");
    const float* base = part + (size_t)kvh * grid_splits * GROUP * PS;
    constexpr size_t SS = (size_t)GROUP * PS;     // floats from one split to the next
    constexpr int MC = 8;
    float* mq = ring;                              // [NQ][NV][6]: m, l, o.xyzw
    static_assert((size_t)NQ * NV * 6 <= (size_t)C::R * C::TILE, "merge groups fit the ring");
    for (int e = ctid; e < NQ * NV; e += CT) {
        const int qg = e / NV, r = e % NV;
        const int h = r / (HD / 4), d4 = (r % (HD / 4)) * 4;
        const float* hb = base + (size_t)h * PS;
        float M = -INFINITY, L = 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = qg; j0 < nsplit; j0 += MC * NQ) {
            float2 ml[MC];
            float4 pv[MC];
#pragma unroll
            for (int i = 0; i < MC; i++) {
                const int j = j0 + i * NQ;
                const float* pj = hb + (size_t)(j < nsplit ? j : 0) * SS;
                ml[i] = j < nsplit ? __ldcg(reinterpret_cast<const float2*>(pj)) : make_float2(-INFINITY, 0.f);
                pv[i] = j < nsplit ? __ldcg(reinterpret_cast<const float4*>(pj + 4 + d4))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float Mc = M;
#pragma unroll
            for (int i = 0; i < MC; i++) Mc = fmaxf(Mc, ml[i].x);
            if (Mc == -INFINITY) continue;
            const float a = M == -INFINITY ? 0.f : expf(M - Mc);   // L, O are 0 before the first split
            L *= a;
            O = make_float4(O.x * a, O.y * a, O.z * a, O.w * a);
#pragma unroll
            for (int i = 0; i < MC; i++)
                if (ml[i].x != -INFINITY) {
                    const float w = expf(ml[i].x - Mc);
                    L = fmaf(ml[i].y, w, L);
                    O = make_float4(fmaf(pv[i].x, w, O.x), fmaf(pv[i].y, w, O.y), fmaf(pv[i].z, w, O.z),
                                    fmaf(pv[i].w, w, O.w));
                }
            M = Mc;
        }
        float* q6 = mq + (size_t)e * 6;
        q6[0] = M;
        q6[1] = L;
        *reinterpret_cast<float2*>(q6 + 2) = make_float2(O.x, O.y);
        *reinterpret_cast<float2*>(q6 + 4) = make_float2(O.z, O.w);
    }
    __syncwarp();   // bar.sync is warp-aligned: reconverge the warp first
    asm volatile("bar.sync 1, %0;" ::"n"(ATTN_CWARPS * 32) : "memory");
    // combine the NQ groups in q order, one output element per thread, in
    // the mt_quantise32 lane layout (a warp holds 32 consecutive columns)
    for (int e = ctid; e < GROUP * HD; e += CT) {
        const int r = e / 4, comp = e % 4;
        float M = -INFINITY;
#pragma unroll
        for (int qg = 0; qg < NQ; qg++) M = fmaxf(M, mq[((size_t)qg * NV + r) * 6]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int qg = 0; qg < NQ; qg++) {
            const float* q6 = mq + ((size_t)qg * NV + r) * 6;
            if (q6[0] == -INFINITY) continue;
            const float w = expf(q6[0] - M);
            L = fmaf(q6[1], w, L);
            O = fmaf(q6[2 + comp], w, O);
        }
        const float val = O / L;
        out[(size_t)kvh * GROUP * HD + e] = val;
        if (xq_out) mt_quantise32(xq_out, n_kv * GROUP * HD, (kvh * GROUP * HD + e) >> 5, lane, val);
    }
    if (ctid == 0) tickets[kvh] = 0u;   // every split has arrived: safe to rearm
}

// part: split partials; tickets: n_kv per-KV-head counters (zero between
// calls); err: the error word (GB_EPOS when pos is outside [0, max_seq)).
// pdl: launch with programmatic stream serialization, so the CTAs start (and
// stream the cached K / V) while the previous kernel finishes.  Only for a
// predecessor that writes neither the caches nor the position (the decode
// step's q/k/v matvec): the producer reads both before griddepcontrol.wait.
template <int HD, int GROUP>
static cudaError_t launch_attn(const float* q, const float* k, const float* v, float* kc, float* vc,
                               const float* cs, const int* d_pos, int n_kv, int max_seq, float* out,
                               float* part, unsigned* tickets, unsigned* err, uint8_t* xq_out, cudaStream_t st,
                               bool pdl) {
    using C = AttnCfg<HD, GROUP>;
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(k_attn_decode<HD, GROUP>), (int)C::SMEM);
    if (e != cudaSuccess) return e;
    const int G = attn_grid_splits(n_kv, max_seq);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_kv * G);
    cfg.blockDim = dim3(ATTN_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn_decode<HD, GROUP>, q, k, v, kc, vc, cs, d_pos, n_kv, max_seq, G, out,
                              part, tickets, err, xq_out);
}

// GB_ATTN_PDL=1 in the environment launches the decode step's attention with
// programmatic dependent launch.
static bool attn_pdl() {
    static const bool v = [] {
        const char* e = getenv("GB_ATTN_PDL");
        return e && e[0] == '1';
    }();
    return v;
}

// Both entry points: pick the instantiation for (head_dim, group).
static int attn_dispatch(const float* q, const float* k, const float* v, float* kc, float* vc, const float* cs,
                         const int* d_pos, int n_heads, int n_kv, int head_dim, int max_seq, float* out,
                         float* part, unsigned* tickets, unsigned* err, cudaStream_t st, uint8_t* xq_out = nullptr,
                         bool pdl = false) {
    const int group = n_heads / n_kv;
    cudaError_t e = cudaErrorInvalidValue;
#define GB_ATTN_CASE(HDV, GV)                                                                                       \
    if (head_dim == HDV && group == GV)                                                                             \
        e = launch_attn<HDV, GV>(q, k, v, kc, vc, cs, d_pos, n_kv, max_seq, out, part, tickets, err, xq_out, st, pdl);
    GB_ATTN_CASE(128, 1) GB_ATTN_CASE(128, 2) GB_ATTN_CASE(128, 4) GB_ATTN_CASE(128, 8)
    GB_ATTN_CASE(64, 1) GB_ATTN_CASE(64, 2) GB_ATTN_CASE(64, 4) GB_ATTN_CASE(64, 8)
#undef GB_ATTN_CASE
    if (e == cudaErrorInvalidValue) return GB_EINVAL;
    return e == cudaSuccess ? GB_OK : GB_ECUDA;
}

// ---------------------------------------------------------------- static scratch
// Scratch of gb_attention_decode_static: a file-scope device array, zero at
// module load.  Layout: words [0, n_kv) split-K tickets (only ever tickets,
// back to zero after every call), word GB_ATTN_STATIC_ERR_WORD the error word,
// partials from byte GB_ATTN_STATIC_PART_OFFSET.
constexpr int GB_ATTN_STATIC_ERR_WORD = 1023;
constexpr size_t GB_ATTN_STATIC_PART_OFFSET = 4096;
static __device__ __align__(256) unsigned char g_attn_static[GB_ATTN_STATIC_BYTES];
static std::mutex g_attn_static_mu;
static void* g_attn_static_addr[64];   // per device, resolved once

static unsigned char* attn_static_scratch(int* rc) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { *rc = GB_ECUDA; return nullptr; }
    if (dev < 0 || dev >= 64) { *rc = GB_ELIMIT; return nullptr; }
    std::lock_guard<std::mutex> lk(g_attn_static_mu);
    if (!g_attn_static_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_attn_static) != cudaSuccess || !p) { *rc = GB_ECUDA; return nullptr; }
        g_attn_static_addr[dev] = p;
    }
    *rc = GB_OK;
    return static_cast<unsigned char*>(g_attn_static_addr[dev]);
}

}  // namespace gb

using namespace gb;

extern "C" size_t gb_attn_workspace_bytes(int n_heads, int n_kv, int head_dim, int max_seq) {
    if (n_kv <= 0 || n_heads % n_kv) return 0;
    const int group = n_heads / n_kv;
    const int G = attn_grid_splits(n_kv, max_seq);
    const size_t part = (size_t)n_kv * G * group * attn_part_stride(head_dim) * sizeof(float);
    return part + (size_t)(n_kv + 1) * sizeof(unsigned);
}

int gb::attention_decode_xq(const float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                            const float* rope_cs, const int* d_pos, int n_heads, int n_kv, int head_dim,
                            int max_seq, float* out, void* ws, uint8_t* xq_out, cudaStream_t st, bool pdl) {
    if (!q || !k || !v || !k_cache || !v_cache || !rope_cs || !d_pos || !out || !ws) return GB_EINVAL;
    if (n_kv <= 0 || n_heads <= 0 || n_heads % n_kv || max_seq <= 0) return GB_EINVAL;
    if (xq_out && (((n_heads * head_dim) % 256) || (reinterpret_cast<uintptr_t>(xq_out) & 15))) return GB_EINVAL;
    const int group = n_heads / n_kv;
    const int G = attn_grid_splits(n_kv, max_seq);
    float* part = static_cast<float*>(ws);
    unsigned* tickets = reinterpret_cast<unsigned*>(part + (size_t)n_kv * G * group * attn_part_stride(head_dim));
    return attn_dispatch(q, k, v, k_cache, v_cache, rope_cs, d_pos, n_heads, n_kv, head_dim, max_seq, out, part,
                         tickets, tickets + n_kv, st, xq_out, pdl && attn_pdl());
}

extern "C" int gb_attention_decode(const float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                                   const float* rope_cs, const int* d_pos, int n_heads, int n_kv, int head_dim,
                                   int max_seq, float* out, void* ws, void* stream) {
    return attention_decode_xq(q, k, v, k_cache, v_cache, rope_cs, d_pos, n_heads, n_kv, head_dim, max_seq, out, ws,
                               nullptr, static_cast<cudaStream_t>(stream), false);
}

extern "C" int gb_attention_decode_static(const float* q, const float* k, const float* v, float* k_cache,
                                          float* v_cache, const float* rope_cs, const int* d_pos, int n_heads,
                                          int n_kv, int head_dim, int max_seq, float* out, void* stream) {
    if (!q || !k || !v || !k_cache || !v_cache || !rope_cs || !d_pos || !out) return GB_EINVAL;
    if (n_kv <= 0 || n_heads <= 0 || n_heads % n_kv || max_seq <= 0) return GB_EINVAL;
    if (n_kv >= GB_ATTN_STATIC_ERR_WORD) return GB_ELIMIT;
    const int group = n_heads / n_kv;
    const int G = attn_grid_splits(n_kv, max_seq);
    const size_t part_bytes = (size_t)n_kv * G * group * attn_part_stride(head_dim) * sizeof(float);
    if (part_bytes > GB_ATTN_STATIC_BYTES - GB_ATTN_STATIC_PART_OFFSET) return GB_ELIMIT;
    int rc;
    unsigned char* base = attn_static_scratch(&rc);
    if (!base) return rc;
    unsigned* words = reinterpret_cast<unsigned*>(base);
    return attn_dispatch(q, k, v, k_cache, v_cache, rope_cs, d_pos, n_heads, n_kv, head_dim, max_seq, out,
                         reinterpret_cast<float*>(base + GB_ATTN_STATIC_PART_OFFSET), words,
                         words + GB_ATTN_STATIC_ERR_WORD, static_cast<cudaStream_t>(stream));
}

extern "C" int gb_attention_static_error(int clear) {
    int rc;
    unsigned char* base = attn_static_scratch(&rc);
    if (!base) return rc;
    unsigned* e = reinterpret_cast<unsigned*>(base) + GB_ATTN_STATIC_ERR_WORD;
    unsigned v = 0;
    if (cudaMemcpy(&v, e, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return GB_ECUDA;
    const unsigned z = 0;
    if (clear && v && cudaMemcpy(e, &z, sizeof(z), cudaMemcpyHostToDevice) != cudaSuccess) return GB_ECUDA;
    return -(int)v;
}
