// gb_chain.cu -- persistent multi-phase matvec for batch-1 decode on sm_100a.
//
// One cooperative launch (one CTA per SM, all co-resident) runs a short
// program of matvec phases, e.g. for one decoder layer boundary
//   wo (+ residual) -> gate/up (RMSNorm fused) -> down (SwiGLU fused,
//   + residual) -> next layer's q/k/v (RMSNorm fused),
// the same operations as the reference's per-layer sequence
// (src/engine/engine.c:433-545 and src/kernels/cuda/cuda_layer_kernels.cu:605-713),
// each phase reading what the previous one wrote.
//
// Why persistent: a kernel per matrix pays its launch, ring fill and tail
// (several microseconds) once per matrix, about 160 times per token.  Here one
// producer lane per CTA streams the weight boxes of ALL phases through a
// shared-memory ring without ever waiting on a phase boundary (weights do not
// depend on x), so HBM keeps streaming while the consumers cross a grid
// barrier and quantise the next x.
//
// Work split: the (matrix, 32-row group, item) sequence of a phase is cut by
// BYTES into one contiguous range per CTA (Q4_K items are one 144-byte block
// x 32 rows, Q6_K items 8 blocks x 32 rows, so the two formats can share a
// phase).  A group shared by CTAs is finished by its first owner at the end of
// that CTA's range: the later owners published their partial rows at the
// start of theirs (release / acquire on a per-group ticket).  Waiting on
// another CTA is safe because the cooperative launch makes every CTA resident.
// The partials are summed in CTA order, so results are deterministic.
//
// Phase barrier: after its last group of phase p a CTA adds 1 to a grid
// counter (release); consumers wait for N (p + 1) arrivals (acquire) before
// reading the next x.  Counters and tickets return to zero before the kernel
// exits.  Every wait is bounded (2 s) and records GB_ETIMEOUT.
#include "gb_mt.cuh"

#include <cstring>
#include <mutex>
#include <vector>

namespace gb {

constexpr int CH_NC = 16;                      // consumer warps
constexpr int CH_THREADS = (CH_NC + 1) * 32;   // + the producer warp
constexpr int CH_NBAR = 8;                     // stage barrier slots
constexpr int CH_NSLOT = CH_NBAR + 2;          // group reduction slots
constexpr int CH_SMEM = 227 * 1024;

// Q4_K stages: one 2-D box of 32 rows x (8 blocks + 16 bytes), row-major in
// shared memory (37.4 KB); split items are single blocks
using ChQ4 = MtQ4KT<1, 8, 8 * GB_Q4K_BYTES + 16>;
using ChQ6 = MtQ6K;          // stages of one 8-block item (53.8 KB)

struct ChMat {
    const void* map;        // device address of the CUtensorMap of the stage boxes
    float* y;
    const float* residual;
    long long ibase;        // first item of the matrix in the phase
    long long bbase;        // its first byte in the phase's byte order
    int fmt;                // 0 = Q4_K, 1 = Q6_K
    int rows;
    int nch;                // items per 32-row group
    long long nitems;
    int gbase;              // first group of the matrix in the phase
};

struct ChPhase {
    ChMat m[CH_MAXM];
    int nm;
    int nb;                 // blocks per row, K = 256 nb
    long long nitems, nbytes;
    int tbase;              // first ticket of the phase
    int s16;                // some matrix is Q6_K: 16-column sums of x
    // x and its transform (MV_X_*), read by the shared quantiser
    const float* x;
    int xmode;
    const float* nw;
    const float* x2;
    float eps;
};

struct alignas(16) ChainDesc {
    ChPhase ph[CH_MAXP];
    int np;
    int ring;               // ring bytes (multiple of 128)
    int kmax;               // largest K of the launch
};

// bytes of one split item in HBM (the byte-balanced split), and of a stage's
// shared-memory slot
__host__ __device__ constexpr int ch_item_bytes(int fmt) { return fmt ? ChQ6::ITEM : GB_Q4K_BYTES * MT_GR; }
__host__ __device__ constexpr int ch_slot_bytes(int fmt, int n) { return fmt ? n * ChQ6::ITEM : ChQ4::STG; }
__host__ __device__ constexpr int ch_item_blocks(int fmt) { return fmt ? ChQ6::IG : ChQ4::IG; }
__host__ __device__ constexpr int ch_stage_items(int fmt) { return fmt ? ChQ6::SI : ChQ4::SI; }

// shared memory after the ring: x | zero line | reductions | counters |
// barriers | the launch descriptor
__host__ __device__ constexpr int ch_tail_bytes(int kmax) {
    return ((mt_xq_bytes(kmax, true) + 15) & ~15) + MT_ZERO + CH_NSLOT * CH_NC * MT_GR * 4 + 64 + 2 * 8 * CH_NBAR +
           64 + (int)((sizeof(ChainDesc) + 15) / 16 * 16) + 16;
}

// ------------------------------------------------------------------ device
// First item of the phase whose first byte is at or after byte b.
__device__ __forceinline__ long long ch_first(const ChPhase& P, long long b) {
    for (int m = 0; m < P.nm; m++) {
        const ChMat& M = P.m[m];
        const long long z = ch_item_bytes(M.fmt);
        const long long u = b <= M.bbase ? 0 : (b - M.bbase + z - 1) / z;
        if (u < M.nitems) return M.ibase + u;
    }
    return P.nitems;
}
// CTA whose byte range [floor(c B / N), floor((c + 1) B / N)) holds item t.
__device__ __forceinline__ int ch_owner(const ChPhase& P, const ChMat& M, long long t, int N) {
    const long long sb = M.bbase + (t - M.ibase) * ch_item_bytes(M.fmt);
    return (int)(((sb + 1) * N - 1) / P.nbytes);
}
// CTA c's range holds at least one item (ranges are cut by bytes, so a CTA
// whose share is smaller than one item may hold none).
__device__ __forceinline__ bool ch_nonempty(const ChPhase& P, int c, int N) {
    return ch_first(P, (long long)c * P.nbytes / N) < ch_first(P, (long long)(c + 1) * P.nbytes / N);
}

// Walk over one CTA's items of a phase, one stage (consecutive items of one
// group, at most a stage's worth) at a time, without divisions per stage.
// The producer and the consumers run the same walk and the same ring
// placement, so stage i means the same boxes to both.
struct ChWalk {
    long long t, t1;   // next item, end of the range
    int m, grp, it;    // position of item t
    __device__ __forceinline__ void start(const ChPhase& P, int c, int N) {
        t = ch_first(P, (long long)c * P.nbytes / N);
        t1 = ch_first(P, (long long)(c + 1) * P.nbytes / N);
        m = 0;
        while (m + 1 < P.nm && t >= P.m[m + 1].ibase) m++;
        const long long u = t < P.nitems ? t - P.m[m].ibase : 0;
        grp = (int)(u / P.m[m].nch);
        it = (int)(u - (long long)grp * P.m[m].nch);
    }
    __device__ __forceinline__ bool more() const { return t < t1; }
    // items in the stage at t
    __device__ __forceinline__ int stage_items(const ChPhase& P) const {
        const ChMat& M = P.m[m];
        long long n = ch_stage_items(M.fmt);
        if (n > M.nch - it) n = M.nch - it;
        if (n > t1 - t) n = t1 - t;
        return (int)n;
    }
    __device__ __forceinline__ void advance(const ChPhase& P, int n) {
        t += n;
        it += n;
        if (it == P.m[m].nch) {
            it = 0;
            if (++grp * P.m[m].nch == P.m[m].nitems) {
                grp = 0;
                m++;
            }
        }
    }
};
// Ring placement: virtual offsets V grow without bound (off = V mod R kept
// alongside); a stage never wraps.
struct ChRing {
    uint32_t V = 0, off = 0;
    __device__ __forceinline__ uint32_t place(uint32_t sz, uint32_t R, uint32_t& soff) {
        if (off + sz > R) {
            V += R - off;
            off = 0;
        }
        const uint32_t v = V;
        soff = off;
        V += sz;
        off += sz;
        return v;
    }
};

constexpr int CH_DESC_SMEM = (sizeof(ChainDesc) + 15) / 16 * 16;

__global__ void __launch_bounds__(CH_THREADS, 1)
k_chain(const ChainDesc* __restrict__ dg, unsigned* __restrict__ sync, float* __restrict__ part,
        unsigned* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x, N = gridDim.x;
    // the launch's descriptor, staged in shared memory (read at every stage)
    const uint32_t R = (uint32_t)__ldg(&dg->ring);
    const int kmax = __ldg(&dg->kmax);
    uint8_t* xq = smem + R;
    uint8_t* zero = xq + ((mt_xq_bytes(kmax, true) + 15) & ~15);
    float* red = reinterpret_cast<float*>(zero + MT_ZERO);
    unsigned* cnt = reinterpret_cast<unsigned*>(red + CH_NSLOT * CH_NC * MT_GR);
    volatile int* abort_f = reinterpret_cast<volatile int*>(cnt + CH_NSLOT);
    const uint32_t bar_full = (sptr(cnt + CH_NSLOT + 4) + 7) & ~7u;
    const uint32_t bar_empty = bar_full + 8 * CH_NBAR;
    ChainDesc* d = reinterpret_cast<ChainDesc*>(smem + ((bar_empty + 8 * CH_NBAR - sptr(smem) + 15) & ~15u));
    const uint32_t sbase = sptr(smem);
    unsigned* const pcount = sync;       // phase arrivals
    unsigned* const ecount = sync + 1;   // exits
    unsigned* const tickets = sync + 2;

    for (int k = threadIdx.x; k < CH_DESC_SMEM / 16; k += blockDim.x)
        reinterpret_cast<uint4*>(d)[k] = __ldg(reinterpret_cast<const uint4*>(dg) + k);
    if (threadIdx.x == 0) {
        for (int s = 0; s < CH_NBAR; s++) {
            mbs_init(bar_full + 8 * s, 1);
            mbs_init(bar_empty + 8 * s, CH_NC);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_f = 0;
    }
    for (int k = threadIdx.x; k < CH_NSLOT; k += blockDim.x) cnt[k] = 0;
    if (threadIdx.x < MT_ZERO / 4) reinterpret_cast<uint32_t*>(zero)[threadIdx.x] = 0;
    __syncthreads();
    const int np = d->np;

    // bounded waits; after the first timeout the CTA stops waiting
    auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        if (*abort_f) return false;
        if (mbs_wait(bar, parity, err)) return true;
        *abort_f = 1;
        return false;
    };

    if (warp == CH_NC) {   // ---- producer: one lane streams every phase's boxes
        if (lane == 0) {
            ChRing ring;
            uint32_t vstart[CH_NBAR];
            int i = 0, rel = 0;   // stages issued; stages [0, rel) known released
            bool ok = true;
            for (int p = 0; p < np && ok; p++) {
                const ChPhase& P = d->ph[p];
                ChWalk w;
                w.start(P, c0, N);
                for (; w.more() && ok; i++) {
                    const int n = w.stage_items(P);
                    const ChMat& M = P.m[w.m];
                    const uint32_t sz = ch_slot_bytes(M.fmt, n);
                    uint32_t soff;
                    const uint32_t vs = ring.place(sz, R, soff);
                    // the barrier slot's previous stage, then every stage that
                    // still holds bytes of [vs, vs + sz) in the ring
                    if (i >= CH_NBAR && rel <= i - CH_NBAR) {
                        ok = wait(bar_empty + 8 * (i % CH_NBAR), ((i / CH_NBAR) - 1) & 1);
                        rel = i - CH_NBAR + 1;
                    }
                    while (ok && rel < i && vstart[rel % CH_NBAR] + R < vs + sz) {
                        ok = wait(bar_empty + 8 * (rel % CH_NBAR), (rel / CH_NBAR) & 1);
                        rel++;
                    }
                    if (!ok) break;
                    vstart[i % CH_NBAR] = vs;
                    const uint32_t fb = bar_full + 8 * (i % CH_NBAR);
                    mbs_expect(fb, sz);
                    // one box per stage: Q6_K one 8-block run (z = run), Q4_K eight
                    // blocks of each row from block it (x = 18 it u64), also for a
                    // stage of fewer items (the extra blocks are not used)
                    if (M.fmt)
                        tma_load_3d(sbase + soff, M.map, 0, w.grp * MT_GR, w.it, fb);
                    else
                        tma_load_3d(sbase + soff, M.map, w.it * ChQ4::IG * (GB_Q4K_BYTES / 8), w.grp * MT_GR, 0, fb);
                    w.advance(P, n);
                }
            }
            // do not retire while a box may still be landing in this CTA's ring
            for (; ok && rel < i; rel++) ok = wait(bar_empty + 8 * (rel % CH_NBAR), (rel / CH_NBAR) & 1);
        }
        return;
    }

    // ---- consumers
    const int tid = threadIdx.x;
    MtLane L4, L6;
    L4.gq = L6.gq = lane >> 2;
    L4.c = L6.c = lane & 3;
    const bool bact = L4.c == (L4.gq >> 1);   // this lane carries a nonzero B fragment
    ChRing ring;
    int i = 0, gi = 0;
    bool ok = true;
    for (int p = 0; p < np; p++) {
        const ChPhase& P = d->ph[p];
        if (p > 0) {   // every CTA's rows of phase p - 1 are written
            if (tid == 0) {
                const unsigned target = (unsigned)(N * p);
                const uint64_t t0 = gtimer();
                while (!*abort_f && ld_acquire(pcount) < target) {
                    if (gtimer() - t0 > MT_WAIT_NS) {
                        atomicExch(err, (unsigned)(-GB_ETIMEOUT));
                        *abort_f = 1;
                    }
                }
            }
            mt_consumer_sync<CH_NC>();
        }
        const int nb = P.nb, K = nb * 256;
        const float rs = P.xmode == MV_X_RMSNORM ? mt_rms_scale<CH_NC>(P.x, K, P.eps, red, tid) : 1.f;
        if (P.s16)
            mt_quantise_x<true>(P, K, xq, tid, CH_NC * 32, rs);
        else
            mt_quantise_x<false>(P, K, xq, tid, CH_NC * 32, rs);
        mt_consumer_sync<CH_NC>();
        L4.xlb = bact ? xq + (L4.gq & 1) * K + ChQ4::XB_LANE * L4.c : zero;
        L6.xlb = bact ? xq + (L6.gq & 1) * K + ChQ6::XB_LANE * L6.c : zero;
        L4.xstr = L6.xstr = bact ? 256 : 0;

        ChWalk w;
        w.start(P, c0, N);
        const long long t0 = w.t, t1 = w.t1;
        float acc_a[2] = {0.f, 0.f}, acc_b[2] = {0.f, 0.f};
        for (; w.more(); i++) {
            const int n = w.stage_items(P);
            const ChMat& M = P.m[w.m];
            uint32_t soff;
            ring.place(ch_slot_bytes(M.fmt, n), R, soff);
            const int s = i % CH_NBAR;
            if (ok) ok = wait(bar_full + 8 * s, (i / CH_NBAR) & 1);
            if (ok) {
                if (M.fmt)
                    ChQ6::consume(smem + soff, w.it * ChQ6::IG, min(nb, (w.it + n) * ChQ6::IG), warp, L6, xq, K,
                                  acc_a, acc_b);
                else
                    ChQ4::consume(smem + soff, w.it * ChQ4::IG, min(nb, (w.it + n) * ChQ4::IG), warp, L4, xq, K,
                                  acc_a, acc_b);
            }
            __syncwarp();
            if (lane == 0) mbs_arrive(bar_empty + 8 * s);
            const int grp = w.grp;
            const bool gdone = w.it + n == M.nch || w.t + n == t1;
            w.advance(P, n);

            if (gdone) {   // ---- this CTA's part of group grp is done
                const int gq = L4.gq, c = L4.c;
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    acc_a[m] += __shfl_xor_sync(0xffffffffu, acc_a[m], 1);
                    acc_a[m] += __shfl_xor_sync(0xffffffffu, acc_a[m], 2);
                    acc_b[m] += __shfl_xor_sync(0xffffffffu, acc_b[m], 1);
                    acc_b[m] += __shfl_xor_sync(0xffffffffu, acc_b[m], 2);
                }
                const int slot = gi % CH_NSLOT;
                float* rw = red + (slot * CH_NC + warp) * MT_GR;
                if (c == 0) {
                    rw[gq] = acc_a[0];
                    rw[gq + 8] = acc_b[0];
                    rw[16 + gq] = acc_a[1];
                    rw[24 + gq] = acc_b[1];
                }
                __syncwarp();
                unsigned tk = 0;
                if (lane == 0) {
                    __threadfence_block();
                    tk = atomicAdd(&cnt[slot], 1u);
                }
                tk = __shfl_sync(0xffffffffu, tk, 0);
                if (tk == CH_NC - 1) {   // last consumer warp: the CTA's rows, summed in warp order
                    __threadfence_block();
                    float v = 0.f;
                    const float* r0 = red + slot * CH_NC * MT_GR + lane;
#pragma unroll
                    for (int w2 = 0; w2 < CH_NC; w2++) v += r0[w2 * MT_GR];
                    __syncwarp();
                    if (lane == 0) cnt[slot] = 0;
                    const long long gs = M.ibase + (long long)grp * M.nch;
                    const int row = grp * MT_GR + lane;
                    if (gs >= t0 && gs + M.nch <= t1) {   // the whole group is this CTA's
                        if (row < M.rows) M.y[row] = v + (M.residual ? __ldcg(M.residual + row) : 0.f);
                    } else {
                        unsigned* tkt = tickets + P.tbase + M.gbase + grp;
                        float* pw = part + ((size_t)(p & 1) * N) * MT_GR;
                        if (gs < t0) {   // a later owner: publish and move on
                            pw[c0 * MT_GR + lane] = v;
                            __threadfence();
                            __syncwarp();
                            if (lane == 0) red_add_release(tkt, 1u);
                        } else {   // the first owner: wait for the later owners' partials
                            const int cl = ch_owner(P, M, gs + M.nch - 1, N);
                            // later owners: cl and every non-empty CTA in between
                            unsigned need = 1;
                            for (int c2 = c0 + 1; c2 < cl; c2++) need += ch_nonempty(P, c2, N) ? 1u : 0u;
                            const uint64_t tw = gtimer();
                            bool got = true;
                            while (ld_acquire(tkt) != need) {
                                if (*abort_f || gtimer() - tw > MT_WAIT_NS) {
                                    if (!*abort_f) atomicExch(err, (unsigned)(-GB_ETIMEOUT));
                                    *abort_f = 1;
                                    got = false;
                                    break;
                                }
                            }
                            float u = v;
                            for (int c2 = c0 + 1; got && c2 <= cl; c2++)
                                if (c2 == cl || ch_nonempty(P, c2, N)) u += __ldcg(pw + c2 * MT_GR + lane);
                            if (got && row < M.rows) M.y[row] = u + (M.residual ? __ldcg(M.residual + row) : 0.f);
                            __syncwarp();
                            if (lane == 0) *tkt = 0u;
                        }
                    }
                }
                acc_a[0] = acc_a[1] = acc_b[0] = acc_b[1] = 0.f;
                gi++;
            }
        }
        mt_consumer_sync<CH_NC>();   // the CTA's rows of phase p are written; x may be replaced
        if (tid == 0 && p + 1 < np) {
            __threadfence();
            red_add_release(pcount, 1u);
        }
    }
    if (tid == 0) {   // the last CTA out resets the counters for the next launch
        __threadfence();
        if (atom_add_acq_rel(ecount, 1u) == (unsigned)(N - 1)) {
            *pcount = 0u;
            *ecount = 0u;
        }
    }
}

// ------------------------------------------------------------------ host
struct ChainSet {
    int nlaunch = 0;
    int grid = 0;
    void* d_maps = nullptr;        // CUtensorMap[nmaps]
    ChainDesc* d_desc = nullptr;   // [nlaunch]
    unsigned* d_sync = nullptr;    // pcount, ecount, tickets
    float* d_part = nullptr;       // [2][grid][MT_GR]
};

bool chain_compatible(int dtype, int cols) {
    if (cols <= 0 || cols % 256) return false;
    if (dtype == GB_DT_Q4_K) return true;
    return dtype == GB_DT_Q6_K && (cols / 256) % 8 == 0;
}

void chain_destroy(ChainSet* cs) {
    if (!cs) return;
    cudaFree(cs->d_maps);
    cudaFree(cs->d_desc);
    cudaFree(cs->d_sync);
    cudaFree(cs->d_part);
    delete cs;
}

int chain_create(const ChPhaseSpec* phases, const int* first, int nlaunch, ChainSet** out) {
    if (!phases || !first || nlaunch <= 0 || !out) return GB_EINVAL;
    *out = nullptr;
    int dev = 0, nsm = 0;
    GB_CUDA_TRY(cudaGetDevice(&dev));
    GB_CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    const int nph = first[nlaunch];
    int nmat = 0;
    for (int q = 0; q < nph; q++) nmat += phases[q].nm;
    std::vector<unsigned char> maps((size_t)nmat * 128);
    std::vector<ChainDesc> desc(nlaunch);
    int mi = 0, max_tickets = 0;
    for (int l = 0; l < nlaunch; l++) {
        const int np = first[l + 1] - first[l];
        if (np <= 0 || np > CH_MAXP) return GB_EINVAL;
        ChainDesc& D = desc[l];
        memset(&D, 0, sizeof(D));
        D.np = np;
        int tick = 0;
        for (int p = 0; p < np; p++) {
            const ChPhaseSpec& ps = phases[first[l] + p];
            ChPhase& P = D.ph[p];
            if (ps.nm <= 0 || ps.nm > CH_MAXM || !ps.x) return GB_EINVAL;
            const int cols = ps.m[0].cols;
            P.nm = ps.nm;
            P.nb = cols / 256;
            P.x = ps.x;
            P.xmode = ps.xf.mode;
            P.nw = ps.xf.mode == MV_X_RMSNORM ? ps.xf.w : nullptr;
            P.x2 = ps.xf.mode == MV_X_SILU_MUL ? ps.xf.x2 : nullptr;
            P.eps = ps.xf.eps;
            if ((P.xmode == MV_X_RMSNORM && !P.nw) || (P.xmode == MV_X_SILU_MUL && !P.x2)) return GB_EINVAL;
            P.tbase = tick;
            long long ib = 0, bb = 0;
            int gb = 0;
            for (int k = 0; k < ps.nm; k++) {
                const ChMatSpec& s = ps.m[k];
                if (s.cols != cols || !chain_compatible(s.dtype, s.cols) || !s.W || !s.y || s.rows <= 0)
                    return GB_EINVAL;
                ChMat& M = P.m[k];
                M.fmt = s.dtype == GB_DT_Q6_K;
                if (M.fmt) P.s16 = 1;
                const bool okm = M.fmt ? mt_encode_view(&maps[(size_t)mi * 128], s.dtype, s.W, s.rows, P.nb, 1)
                                       : mt_encode_rows(&maps[(size_t)mi * 128], s.W, s.rows, P.nb, ChQ4::RP / 8);
                if (!okm) return GB_EINVAL;
                M.map = reinterpret_cast<const void*>((uintptr_t)mi * 128);   // offset; rebased below
                mi++;
                M.y = s.y;
                M.residual = s.residual;
                M.rows = s.rows;
                M.nch = P.nb / ch_item_blocks(M.fmt);
                const int groups = (s.rows + MT_GR - 1) / MT_GR;
                M.nitems = (long long)groups * M.nch;
                M.ibase = ib;
                M.bbase = bb;
                M.gbase = gb;
                ib += M.nitems;
                bb += M.nitems * ch_item_bytes(M.fmt);
                gb += groups;
            }
            P.nitems = ib;
            P.nbytes = bb;
            tick += gb;
            D.kmax = std::max(D.kmax, cols);
        }
        max_tickets = std::max(max_tickets, tick);
        const int ring = (CH_SMEM - ch_tail_bytes(D.kmax)) & ~127;
        if (ring < 2 * ChQ6::STG) return GB_ELIMIT;
        D.ring = ring;
    }
    ChainSet* cs = new ChainSet;
    cs->nlaunch = nlaunch;
    cs->grid = nsm;
    bool okm = cudaMalloc(&cs->d_maps, maps.size()) == cudaSuccess &&
               cudaMalloc(reinterpret_cast<void**>(&cs->d_desc), sizeof(ChainDesc) * nlaunch) == cudaSuccess &&
               cudaMalloc(reinterpret_cast<void**>(&cs->d_sync), sizeof(unsigned) * (2 + max_tickets)) == cudaSuccess &&
               cudaMalloc(reinterpret_cast<void**>(&cs->d_part), sizeof(float) * 2 * nsm * MT_GR) == cudaSuccess;
    if (!okm) {
        chain_destroy(cs);
        return GB_ENOMEM;
    }
    for (auto& D : desc)
        for (int p = 0; p < D.np; p++)
            for (int k = 0; k < D.ph[p].nm; k++) {
                ChMat& M = D.ph[p].m[k];
                M.map = static_cast<const char*>(cs->d_maps) + reinterpret_cast<uintptr_t>(M.map);
            }
    if (cudaMemcpy(cs->d_maps, maps.data(), maps.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(cs->d_desc, desc.data(), sizeof(ChainDesc) * nlaunch, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(cs->d_sync, 0, sizeof(unsigned) * (2 + max_tickets)) != cudaSuccess) {
        chain_destroy(cs);
        return GB_ECUDA;
    }
    *out = cs;
    return GB_OK;
}

int chain_launch(const ChainSet* cs, int i, unsigned* err, cudaStream_t st) {
    if (!cs || i < 0 || i >= cs->nlaunch || !err) return GB_EINVAL;
    static unsigned configured = 0;
    static std::mutex mu;
    int dev = 0;
    GB_CUDA_TRY(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!(configured & (1u << (dev & 31)))) {
            GB_CUDA_TRY(cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, CH_SMEM));
            configured |= 1u << (dev & 31);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs->grid);
    cfg.blockDim = dim3(CH_THREADS);
    cfg.dynamicSmemBytes = CH_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GB_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_chain, static_cast<const ChainDesc*>(cs->d_desc + i), cs->d_sync,
                                   cs->d_part, err));
    return GB_OK;
}

}  // namespace gb
