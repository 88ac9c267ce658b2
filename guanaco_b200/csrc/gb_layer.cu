// gb_layer.cu -- layer glue kernels and the device-resident decode model.
//
// The model runs forward() of src/engine/engine.c:559-594 for one token
// (T = 1) entirely on the device:
//   embedding row dequant                        engine.c:214-283
//   per layer (engine.c:353-554):
//     rmsnorm -> Wq, Wk, Wv -> RoPE + KV append + attention -> Wo (+residual)
//     -> rmsnorm -> gate, up -> silu(gate)*up -> down (+residual)
//   final rmsnorm -> lm_head -> greedy argmax (tokenizer.c:175-185)
// The whole step is captured once into a CUDA graph (token and position are
// read from device memory) and replayed per token.
#include "gb_common.cuh"
#include "gb_internal.h"

#include <algorithm>

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

namespace gb {

static std::mutex g_dev_mu;

int sm_count() {
    static std::atomic<int> counts[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 1;
    if (dev < 64) {
        const int c = counts[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 1;
    if (n > GB_MAX_SMS) n = GB_MAX_SMS;
    if (dev < 64) counts[dev].store(n, std::memory_order_relaxed);
    return n;
}

cudaError_t set_smem_once(const void* func, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::set<std::pair<const void*, int>> done;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (done.count({func, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({func, dev});
    return e;
}

// ---------------------------------------------------------------- glue kernels
__device__ __forceinline__ float block_sum_1024(float v, float* sh) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.f;
    if (warp == 0) v = warp_sum(v);
    if (threadIdx.x == 0) sh[32] = v;
    __syncthreads();
    const float r = sh[32];
    __syncthreads();
    return r;
}

// out = w * (x * r), r = 1/sqrt(sum(x^2)/n + eps)  (kernels_cpu.c:242-263),
// row blockIdx.x of n-element rows
__global__ void __launch_bounds__(1024) k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w,
                                                  float* __restrict__ out, int n, float eps) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // successors may start their weight prefetch
    x += (size_t)blockIdx.x * n;
    out += (size_t)blockIdx.x * n;
    __shared__ float sh[33];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum_1024(ss, sh);
    const float r = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = __fmul_rn(w ? w[i] : 1.0f, __fmul_rn(x[i], r));
}

// gate = (gate * (1/(1+exp(-gate)))) * up  (kernels_cpu.c:323-336, 381-384)
__global__ void k_silu_mul(float* __restrict__ g, const float* __restrict__ u, int n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // successors may start their weight prefetch
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float x = g[i];
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    g[i] = __fmul_rn(__fmul_rn(x, sig), u[i]);
}

// Multi-CTA argmax for long vectors (the output head): CTA c scans the
// contiguous chunk [c n / G, (c + 1) n / G) and writes its (max, first index);
// the last CTA to finish (ticket) merges the chunks in index order, so the
// first maximum wins as in sample_greedy (tokenizer.c:175-185).
struct ArgPart { float v; int i; };
constexpr int AM_MAX_CTAS = 148;   // split-argmax CTAs at most (its workspace size)
constexpr size_t AM_WS_BYTES = AM_MAX_CTAS * sizeof(ArgPart) + 16;
__global__ void __launch_bounds__(1024) k_argmax_split(const float* __restrict__ x, int n, int* __restrict__ out,
                                                       ArgPart* __restrict__ part, unsigned* __restrict__ ticket,
                                                       ArgPart* __restrict__ result, int off) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // successors may start their weight prefetch
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ bool last;
    const int G = gridDim.x, c = blockIdx.x;
    const int lo = (int)((long long)c * n / G), hi = (int)((long long)(c + 1) * n / G);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = x[i];
        if (v > bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        part[c].v = bv;
        part[c].i = bi;
        __threadfence();
        last = atomicAdd(ticket, 1u) == (unsigned)(G - 1);
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    float mv = -INFINITY;
    int mi = 0x7fffffff;
    for (int k = 0; k < G; k++) {   // chunk order = index order: strict > keeps the first maximum
        const float v = __ldcg(&part[k].v);
        const int i = __ldcg(&part[k].i);
        if (v > mv || (v == mv && i < mi)) { mv = v; mi = i; }
    }
    mi = mi == 0x7fffffff ? 0 : mi;
    *out = mi + off;
    if (result) {   // (max, global index) for the tensor-parallel merge
        result->v = mv;
        result->i = mi + off;
    }
    *ticket = 0u;
}

// First index of the maximum, strict > (ties keep the lower index).
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ x, int n, int* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) *out = bi == 0x7fffffff ? 0 : bi;
    }
}

// Embedding rows of d_token[0 .. gridDim.y) (engine.c:214-283): F32 copy,
// Q8_0 q*scale, Q4_K d1*q - m1 -- bit-exact with the reference dequantiser.
// Row y of out is token y's (a decode step has one row).
__global__ void k_embed(const void* __restrict__ emb, int dtype, const int* __restrict__ d_token, int vocab, int H,
                        float* __restrict__ out, unsigned* __restrict__ err, unsigned long long* __restrict__ step) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // successors may start their weight prefetch
    if (step && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *step += 1;   // epochs of this step's exchanges
    const int tok = d_token[blockIdx.y];
    out += (size_t)blockIdx.y * H;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && err) atomicExch(err, (unsigned)(-GB_EINVAL));
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
        if (dtype == GB_DT_F32) {
            out[i] = static_cast<const float*>(emb)[(size_t)tok * H + i];
        } else if (dtype == GB_DT_Q8_0) {
            const uint8_t* blk = static_cast<const uint8_t*>(emb) + ((size_t)tok * (H / 32) + i / 32) * GB_Q80_BYTES;
            out[i] = __fmul_rn((float)(int8_t)blk[2 + (i & 31)], f16_bits_to_f32(blk[0] | (blk[1] << 8)));
        } else {   // Q4_K
            const uint8_t* blk = static_cast<const uint8_t*>(emb) + ((size_t)tok * (H / 256) + i / 256) * GB_Q4K_BYTES;
            const int w = i & 255, g = w >> 6, hi = (w >> 5) & 1, l = w & 31, j = 2 * g + hi;
            const uint8_t* s = blk + 4;
            uint32_t sc, mn;
            if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
            else { sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
            const float d_all = f16_bits_to_f32(blk[0] | (blk[1] << 8));
            const float min_all = f16_bits_to_f32(blk[2] | (blk[3] << 8));
            const uint8_t qb = blk[16 + 32 * g + l];
            const uint32_t q = hi ? (qb >> 4) : (qb & 0xF);
            out[i] = __fsub_rn(__fmul_rn(__fmul_rn(d_all, (float)sc), (float)q), __fmul_rn(min_all, (float)mn));
        }
    }
}

__global__ void k_set_int(int* p, int v) { *p = v; }
// Feed the greedy token back and move to the next position; record it.
__global__ void k_advance(int* tok, const int* next, int* pos, int* out, int* count) {
    *tok = *next;
    *pos += 1;
    if (out) out[*count] = *next;
    *count += 1;
}

// ---------------------------------------------------------------- tensor parallel exchanges
// Every rank owns a receive buffer in its own HBM; the others write into it
// over NVLink through CUDA IPC mappings.  Layout (world <= 8, H floats):
//   slots [2][world][H] {value bits, epoch} | results [2][world] ArgPart |
//   flags [2][world] u32
// Exchange e of a step gets epoch = step * calls + e + 1 (unique, the same on
// every rank); it uses parity e & 1, so a rank one exchange ahead never
// overwrites data a peer is still reading.  Slots: a sender writes each
// value together with its epoch in one 8-byte store; a reader waits until
// the epoch tag matches (bounded: 2 s, then GB_ETIMEOUT in the error word).
// The hidden-state exchanges normally run inside the matvecs (MvTp: wo /
// ffn_down push their rows, the next RMSNorm matvec sums them);
// k_tp_allreduce does both sides as its own launch for shapes those kernels
// do not take.  The argmax exchange publishes one (max, index) per rank and
// releases flag[parity][sender] = epoch after a system-scope fence.
__device__ __forceinline__ size_t tp_slots_bytes(int world, int H) { return (size_t)2 * world * H * sizeof(uint2); }
__device__ __forceinline__ unsigned* tp_flags(void* base, int world, int H) {
    return reinterpret_cast<unsigned*>(static_cast<char*>(base) + tp_slots_bytes(world, H) + 2 * world * sizeof(ArgPart));
}
__device__ __forceinline__ ArgPart* tp_results(void* base, int world, int H) {
    return reinterpret_cast<ArgPart*>(static_cast<char*>(base) + tp_slots_bytes(world, H));
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t tp_gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// wait until flags[i] has reached ep (wrap-safe); false after 2 s
__device__ bool tp_wait_flag(const unsigned* flag, unsigned ep) {
    if ((int)(ld_acquire_sys(flag) - ep) >= 0) return true;
    const uint64_t t0 = tp_gtimer();
    while ((int)(ld_acquire_sys(flag) - ep) < 0)
        if (tp_gtimer() - t0 > 2000000000ull) return false;
    return true;
}
__device__ __forceinline__ void tp_ll_store(uint2* p, float v, unsigned tag) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}
// value of slot p once its tag is ep; false after 2 s
__device__ __forceinline__ bool tp_ll_wait(const uint2* p, unsigned ep, float& v) {
    uint32_t x, t;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(t) : "l"(p) : "memory");
    if (t != ep) {
        const uint64_t t0 = tp_gtimer();
        do {
            if (tp_gtimer() - t0 > 2000000000ull) return false;
            asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(t) : "l"(p) : "memory");
        } while (t != ep);
    }
    v = __uint_as_float(x);
    return true;
}

// h_out = h_in + sum over ranks (in rank order) of every rank's partial.
// Grid = world CTAs: CTA p pushes this rank's partial to peer p, then
// reduces slice p from this rank's own buffer.
__global__ void __launch_bounds__(512) k_tp_allreduce(const float* __restrict__ part, const float* __restrict__ h_in,
                                                      float* __restrict__ h_out, int H, int rank, int world,
                                                      void* const* __restrict__ peers,
                                                      const unsigned long long* __restrict__ step, int calls,
                                                      int call, unsigned* __restrict__ err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // successors may start their weight prefetch
    const unsigned ep = (unsigned)(*step * (unsigned long long)calls + call + 1);
    const int par = ep & 1, p = blockIdx.x, tid = threadIdx.x;
    uint2* dst = static_cast<uint2*>(peers[p]) + ((size_t)par * world + rank) * H;
    for (int i = tid; i < H; i += blockDim.x) tp_ll_store(dst + i, part[i], ep);
    const uint2* slots = static_cast<const uint2*>(peers[rank]) + (size_t)par * world * H;
    const int lo = (int)((long long)p * H / world), hi = (int)((long long)(p + 1) * H / world);
    bool ok = true;
    for (int i = lo + tid; i < hi; i += blockDim.x) {
        float sum = 0.f;
        for (int q = 0; q < world; q++) {
            float v = 0.f;
            if (ok && !tp_ll_wait(slots + (size_t)q * H + i, ep, v)) {
                ok = false;
                atomicExch(err, (unsigned)(-GB_ETIMEOUT));
            }
            sum += v;
        }
        h_out[i] = h_in[i] + sum;
    }
}

// Greedy token over the vocabulary shards: every rank publishes its shard's
// (max, global index) and takes the best in rank order (shards are in index
// order, so ties keep the lowest index, as sample_greedy).
__global__ void k_tp_argmax(const ArgPart* __restrict__ mine_res, int* __restrict__ out, int H, int rank, int world,
                            void* const* __restrict__ peers, const unsigned long long* __restrict__ step, int calls,
                            int call, unsigned* __restrict__ err) {
    const unsigned ep = (unsigned)(*step * (unsigned long long)calls + call + 1);
    const int par = ep & 1, t = threadIdx.x;
    if (t < world) {
        tp_results(peers[t], world, H)[par * world + rank] = *mine_res;
        __threadfence_system();
        st_release_sys(tp_flags(peers[t], world, H) + par * world + rank, ep);
    }
    __syncwarp();
    void* mine = peers[rank];
    if (t < world && !tp_wait_flag(tp_flags(mine, world, H) + par * world + t, ep))
        atomicExch(err, (unsigned)(-GB_ETIMEOUT));
    __syncwarp();
    if (t != 0) return;
    const ArgPart* r = tp_results(mine, world, H) + par * world;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = 0; q < world; q++) {
        const float v = __ldcg(&r[q].v);
        const int i = __ldcg(&r[q].i);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    *out = bi == 0x7fffffff ? 0 : bi;
}

}  // namespace gb

using namespace gb;

// ---------------------------------------------------------------- glue C ABI
extern "C" int gb_rmsnorm(const float* x, const float* w, float* out, int n, float eps, void* stream) {
    if (!x || !out || n <= 0) return GB_EINVAL;
    k_rmsnorm<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out, n, eps);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
extern "C" int gb_silu_mul(float* gate, const float* up, int n, void* stream) {
    if (!gate || !up || n <= 0) return GB_EINVAL;
    k_silu_mul<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, n);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
extern "C" int gb_argmax(const float* x, int n, int* d_out, void* stream) {
    if (!x || !d_out || n <= 0) return GB_EINVAL;
    k_argmax<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, n, d_out);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}

extern "C" void gb_host_rope_table(float* h_cs, int max_seq, int head_dim, float theta);  // gb_host.c

extern "C" int gb_rope_table(float* cs, int max_seq, int head_dim, float theta, void* stream) {
    if (!cs || max_seq <= 0 || head_dim <= 0 || (head_dim & 1)) return GB_EINVAL;
    const size_t n = (size_t)max_seq * head_dim;
    float* h = nullptr;
    if (cudaMallocHost(&h, n * sizeof(float)) != cudaSuccess) return GB_ENOMEM;
    gb_host_rope_table(h, max_seq, head_dim, theta);
    cudaError_t e = cudaMemcpyAsync(cs, h, n * sizeof(float), cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    cudaFreeHost(h);
    return e == cudaSuccess ? GB_OK : GB_ECUDA;
}

extern "C" const char* gb_version(void) { return "guanaco_b200 0.1 (sm_100a)"; }
extern "C" int gb_device_sm_count(void) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return n;
}

// ---------------------------------------------------------------- model
struct gb_model {
    gb_model_config c;
    int kv_dim = 0;                   // local KV width (nkv * head_dim)
    // tensor parallelism: this rank's slice of the model (rank, world)
    int rank = 0, world = 1;
    int nh = 0, nkv = 0;              // local q / kv heads
    int ff = 0, ff_pad = 0;           // local FFN rows; padded width of the gate / up buffers
    bool pad_down = false;            // gb_model_synthesize: Q6_K ffn_down rows padded to ff_pad columns
    int vocab_l = 0, vocab_off = 0;   // output-head rows of this rank
    void* comm = nullptr;             // exchange buffer (world > 1)
    size_t comm_bytes = 0;
    void** d_peers = nullptr;         // device array of the world exchange buffers
    void* peer_open[8] = {};          // IPC mappings opened by this rank
    bool comm_ready = false;
    unsigned long long* d_step = nullptr;
    float* part = nullptr;            // local partial of wo / ffn_down
    unsigned* tp_ready = nullptr;     // per-CTA slice flags of the in-matvec exchanges (zeroed)
    ArgPart* am_res = nullptr;        // local (max, index) of the output head
    TpCtx tp;
    std::vector<const void*> w;       // [n_layers * 7]
    std::vector<int> dt;              // [n_layers * 7]
    std::vector<const float*> ra, rf; // [n_layers]
    const void* emb = nullptr;
    int emb_dt = GB_DT_Q4_K;
    const float* rms_final = nullptr;
    const void* lm = nullptr;
    int lm_dt = GB_DT_Q6_K;
    std::vector<MvPlan> plan;         // [n_layers * 7] prepared matvecs
    MvPlan lm_plan;
    void* mv_ws = nullptr;            // shared matvec workspace (zeroed)
    size_t mv_ws_size = 0;
    std::vector<void*> owned;         // allocations freed with the model

    float *kc = nullptr, *vc = nullptr, *rope = nullptr;
    float* hidden2 = nullptr;         // tensor parallel: second hidden-state buffer (exchanges ping-pong)
    uint8_t* swq = nullptr;           // SwiGLU product quantised for ffn_down (zeroed)
    uint8_t* aq = nullptr;            // attention output quantised for wo
    unsigned* swq_tk = nullptr;       // its pair tickets (zero)
    void* attn_ws = nullptr;
    float *hidden = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *gate = nullptr, *up = nullptr, *logits = nullptr;
    unsigned* err = nullptr;
    int *d_tok = nullptr, *d_pos = nullptr, *d_next = nullptr;
    int* io = nullptr;                // device {token, pos, next, error}: d_tok .. err point into it
    int* h_io = nullptr;              // pinned {token, pos, next, error}
    cudaStream_t stream = nullptr;

    cudaGraphExec_t exec = nullptr;
    const void* key[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    cudaGraphExec_t gen_exec = nullptr;   // step + advance, for gb_model_generate
    const void* gen_key[4] = {nullptr, nullptr, nullptr, nullptr};
    int* d_count = nullptr;
    void* am_ws = nullptr;            // argmax partials + ticket (zeroed)
    // prefill activations for up to pf_cap tokens (allocated by the first
    // prefill, grown when a longer chunk arrives, freed with the model)
    void* pf = nullptr;
    int pf_cap = 0;
    int* pf_tok = nullptr;            // device copy of a host prompt
    int pf_tok_cap = 0;
    // prefill: a second stream for the wk / wv GEMMs, which run beside wq
    // (fork / join events recorded on the caller's stream)
    cudaStream_t pf_side = nullptr;
    cudaEvent_t pf_fork = nullptr, pf_join = nullptr;
};

static void* dalloc(gb_model* m, size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    m->owned.push_back(p);
    return p;
}

static void invalidate_graph(gb_model* m);

// Exchange buffer of one rank: slots [2][world][H] {value, epoch} pairs,
// results [2][world], flags [2][world] u32 (see k_tp_allreduce).
static size_t tp_comm_bytes(int world, int H) {
    return (size_t)2 * world * H * sizeof(uint2) + 2 * world * sizeof(ArgPart) + 2 * world * sizeof(unsigned);
}

// Form of the hidden-state exchanges inside the matvecs: with few ranks every
// CTA reads all ranks' slots itself (direct; world x H x 8 bytes of L2 reads
// per CTA, no grid-wide wait); with more, each CTA reduces one slice and the
// CTAs meet on per-CTA flags (slice; the slots are read once).
// GB_TP_EXCHANGE=direct|slice in the environment overrides the choice.
static bool tp_slice_exchange(int world) {
    const char* e = getenv("GB_TP_EXCHANGE");
    if (e && !strcmp(e, "direct")) return false;
    if (e && !strcmp(e, "slice")) return true;
    return world > 2;
}

extern "C" gb_model* gb_model_create_tp(const gb_model_config* cfg, int rank, int world) {
    if (!cfg) return nullptr;
    const gb_model_config& c = *cfg;
    if (c.hidden_dim <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
        c.head_dim * c.n_heads != c.hidden_dim || c.n_layers <= 0 || c.ff_dim <= 0 || c.vocab_size <= 0 ||
        c.max_seq <= 0)
        return nullptr;
    // shards: heads by rank (KV heads too), FFN rows in 256-column blocks,
    // wo columns in whole blocks, vocabulary rows by rank
    if (world < 1 || world > 8 || rank < 0 || rank >= world) return nullptr;
    if (world > 1 && (c.n_kv_heads % world || c.ff_dim % (256 * world) ||
                      (c.n_heads / world * c.head_dim) % 256 || c.hidden_dim % 4))
        return nullptr;
    gb_model* m = new gb_model();
    m->c = c;
    m->rank = rank;
    m->world = world;
    m->nh = c.n_heads / world;
    m->nkv = c.n_kv_heads / world;
    m->ff = c.ff_dim / world;
    // a Q6_K ffn_down shard (and a synthesised one-GPU ffn_down) keeps its
    // rows at 8-block multiples (zero blocks after the FFN columns) so its
    // tensor map has a 16-byte stride; the gate / up buffers carry the
    // matching zero tail
    m->ff_pad = (m->ff + 2047) / 2048 * 2048;
    m->vocab_off = (int)((long long)rank * c.vocab_size / world);
    m->vocab_l = (int)((long long)(rank + 1) * c.vocab_size / world) - m->vocab_off;
    m->kv_dim = m->nkv * c.head_dim;
    m->w.assign((size_t)c.n_layers * GB_NMAT, nullptr);
    m->dt.assign((size_t)c.n_layers * GB_NMAT, GB_DT_Q4_K);
    m->plan.assign((size_t)c.n_layers * GB_NMAT, MvPlan{});
    m->ra.assign(c.n_layers, nullptr);
    m->rf.assign(c.n_layers, nullptr);
    const size_t kv_elems = (size_t)c.n_layers * m->kv_dim * c.max_seq;
    const int H = c.hidden_dim, QD = m->nh * c.head_dim, FP = m->ff_pad;
    bool ok = true;
    ok &= (m->kc = (float*)dalloc(m, kv_elems * 4)) != nullptr;
    ok &= (m->vc = (float*)dalloc(m, kv_elems * 4)) != nullptr;
    ok &= (m->rope = (float*)dalloc(m, (size_t)c.max_seq * c.head_dim * 4)) != nullptr;
    const size_t ws = gb_attn_workspace_bytes(m->nh, m->nkv, c.head_dim, c.max_seq);
    ok &= ws > 0 && (m->attn_ws = dalloc(m, ws)) != nullptr;
    ok &= (m->hidden = (float*)dalloc(m, (size_t)H * 4)) != nullptr;
    ok &= (m->xn = (float*)dalloc(m, (size_t)(H > FP ? H : FP) * 4)) != nullptr;
    ok &= (m->q = (float*)dalloc(m, (size_t)QD * 4)) != nullptr;
    ok &= (m->k = (float*)dalloc(m, (size_t)m->kv_dim * 4)) != nullptr;
    ok &= (m->v = (float*)dalloc(m, (size_t)m->kv_dim * 4)) != nullptr;
    ok &= (m->attn = (float*)dalloc(m, (size_t)QD * 4)) != nullptr;
    ok &= (m->gate = (float*)dalloc(m, (size_t)FP * 4)) != nullptr;
    ok &= (m->up = (float*)dalloc(m, (size_t)FP * 4)) != nullptr;
    const size_t swq_bytes = FP % 256 ? 0 : (size_t)FP * 7 / 2;   // x0, x1, x2, per-64 scales and sums, 16-column sums
    if (swq_bytes) {
        ok &= (m->swq = (uint8_t*)dalloc(m, swq_bytes)) != nullptr;
        ok &= (m->swq_tk = (unsigned*)dalloc(m, (size_t)FP / 32 * sizeof(unsigned))) != nullptr;
    }
    // wo's input quantised by the attention launch (same layout)
    if (QD % 256 == 0) ok &= (m->aq = (uint8_t*)dalloc(m, (size_t)QD * 7 / 2)) != nullptr;
    ok &= (m->logits = (float*)dalloc(m, (size_t)m->vocab_l * 4)) != nullptr;
    // the host-facing words share one block: gb_model_decode_host sends
    // {token, pos} in one copy and reads {next, error} back in one copy
    ok &= (m->io = (int*)dalloc(m, 64)) != nullptr;
    if (m->io) {
        m->d_tok = m->io;
        m->d_pos = m->io + 1;
        m->d_next = m->io + 2;
        m->err = reinterpret_cast<unsigned*>(m->io + 3);
    }
    ok &= (m->d_count = (int*)dalloc(m, 16)) != nullptr;
    ok &= (m->am_ws = dalloc(m, AM_WS_BYTES)) != nullptr;
    ok &= (m->d_step = (unsigned long long*)dalloc(m, 16)) != nullptr;
    ok &= (m->am_res = (ArgPart*)dalloc(m, 16)) != nullptr;
    if (world > 1) {
        m->comm_bytes = tp_comm_bytes(world, H);
        ok &= (m->part = (float*)dalloc(m, (size_t)H * 4)) != nullptr;
        ok &= (m->hidden2 = (float*)dalloc(m, (size_t)H * 4)) != nullptr;
        ok &= (m->tp_ready = (unsigned*)dalloc(m, GB_MAX_SMS * sizeof(unsigned))) != nullptr;
        ok &= (m->d_peers = (void**)dalloc(m, 8 * sizeof(void*))) != nullptr;
        // the exchange buffer gets its own allocation: it is shared with the
        // peers through cudaIpcGetMemHandle
        if (ok && cudaMalloc(&m->comm, m->comm_bytes) != cudaSuccess) { m->comm = nullptr; ok = false; }
    }
    ok &= cudaMallocHost(&m->h_io, 4 * sizeof(int)) == cudaSuccess;
    ok &= cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess;
    // zero in stream order, then wait: decode may run on any stream
    if (ok) ok &= cudaMemsetAsync(m->kc, 0, kv_elems * 4, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->vc, 0, kv_elems * 4, m->stream) == cudaSuccess;
    if (ok) ok &= cudaMemsetAsync(m->attn_ws, 0, ws, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->io, 0, 64, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->am_ws, 0, AM_WS_BYTES, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->d_step, 0, 16, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->gate, 0, (size_t)FP * 4, m->stream) == cudaSuccess &&
                  cudaMemsetAsync(m->up, 0, (size_t)FP * 4, m->stream) == cudaSuccess;
    if (ok && m->swq) ok &= cudaMemsetAsync(m->swq, 0, swq_bytes, m->stream) == cudaSuccess &&
                            cudaMemsetAsync(m->swq_tk, 0, (size_t)FP / 32 * sizeof(unsigned), m->stream) == cudaSuccess;
    if (ok && m->comm) ok &= cudaMemsetAsync(m->comm, 0, m->comm_bytes, m->stream) == cudaSuccess;
    if (ok && m->tp_ready) ok &= cudaMemsetAsync(m->tp_ready, 0, GB_MAX_SMS * sizeof(unsigned), m->stream) == cudaSuccess;
    if (ok) ok &= gb_rope_table(m->rope, c.max_seq, c.head_dim, c.rope_theta, m->stream) == GB_OK;
    if (ok) ok &= cudaStreamSynchronize(m->stream) == cudaSuccess;
    if (!ok) {
        gb_model_destroy(m);
        return nullptr;
    }
    m->tp.rank = rank;
    m->tp.world = world;
    m->tp.d_peers = m->d_peers;
    m->tp.d_step = m->d_step;
    m->tp.calls = 2 * c.n_layers + 1;
    m->tp.err = m->err;
    m->tp.ready = tp_slice_exchange(world) ? m->tp_ready : nullptr;
    m->tp.part = m->part;
    m->tp.h[0] = m->hidden;
    m->tp.h[1] = m->hidden2;
    return m;
}

extern "C" gb_model* gb_model_create(const gb_model_config* cfg) { return gb_model_create_tp(cfg, 0, 1); }

extern "C" int gb_model_comm_handle(gb_model* m, void* handle) {
    if (!m || !handle || m->world < 2 || !m->comm) return GB_EINVAL;
    cudaIpcMemHandle_t h;
    GB_CUDA_TRY(cudaIpcGetMemHandle(&h, m->comm));
    memcpy(handle, &h, sizeof(h));
    return GB_OK;
}

extern "C" int gb_model_comm_open(gb_model* m, const void* handles) {
    if (!m || !handles || m->world < 2 || !m->comm || m->comm_ready) return GB_EINVAL;
    void* peers[8] = {};
    for (int q = 0; q < m->world; q++) {
        if (q == m->rank) {
            peers[q] = m->comm;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)q * GB_IPC_HANDLE_BYTES, sizeof(h));
        if (cudaIpcOpenMemHandle(&peers[q], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            for (int j = 0; j < q; j++)
                if (j != m->rank && peers[j]) cudaIpcCloseMemHandle(peers[j]);
            return GB_ECUDA;
        }
    }
    for (int q = 0; q < m->world; q++) m->peer_open[q] = q == m->rank ? nullptr : peers[q];
    GB_CUDA_TRY(cudaMemcpy(m->d_peers, peers, sizeof(peers), cudaMemcpyHostToDevice));
    m->comm_ready = true;
    invalidate_graph(m);
    return GB_OK;
}

extern "C" int gb_model_tp_info(const gb_model* m, int* rank, int* world, int* vocab_off, int* vocab_rows) {
    if (!m) return GB_EINVAL;
    if (rank) *rank = m->rank;
    if (world) *world = m->world;
    if (vocab_off) *vocab_off = m->vocab_off;
    if (vocab_rows) *vocab_rows = m->vocab_l;
    return GB_OK;
}

extern "C" void gb_model_destroy(gb_model* m) {
    if (!m) return;
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->gen_exec) cudaGraphExecDestroy(m->gen_exec);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (void* p : m->peer_open)
        if (p) cudaIpcCloseMemHandle(p);
    if (m->comm) cudaFree(m->comm);
    for (void* p : m->owned) cudaFree(p);
    if (m->pf_side) cudaStreamSynchronize(m->pf_side);
    if (m->pf) cudaFree(m->pf);
    if (m->pf_tok) cudaFree(m->pf_tok);
    if (m->pf_fork) cudaEventDestroy(m->pf_fork);
    if (m->pf_join) cudaEventDestroy(m->pf_join);
    if (m->pf_side) cudaStreamDestroy(m->pf_side);
    if (m->h_io) cudaFreeHost(m->h_io);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

static void invalidate_graph(gb_model* m) {
    if (m->exec) { cudaGraphExecDestroy(m->exec); m->exec = nullptr; }
    if (m->gen_exec) { cudaGraphExecDestroy(m->gen_exec); m->gen_exec = nullptr; }
}

static void mat_shape(const gb_model* m, int which, int dtype, int* rows, int* cols);
static void invalidate_graph(gb_model* m);

extern "C" int gb_model_set_matrix(gb_model* m, int layer, int which, int dtype, const void* d_w) {
    if (!m || layer < 0 || layer >= m->c.n_layers || which < 0 || which >= GB_NMAT || !d_w) return GB_EINVAL;
    if (dtype != GB_DT_Q4_K && dtype != GB_DT_Q6_K && dtype != GB_DT_Q8_0 && dtype != GB_DT_Q5_K &&
        dtype != GB_DT_F16)
        return GB_EINVAL;
    int rows, cols;
    mat_shape(m, which, dtype, &rows, &cols);
    MvPlan p;
    const int rc = mv_plan(&p, dtype, d_w, rows, cols);
    if (rc) return rc;
    m->w[(size_t)layer * GB_NMAT + which] = d_w;
    m->dt[(size_t)layer * GB_NMAT + which] = dtype;
    m->plan[(size_t)layer * GB_NMAT + which] = p;
    invalidate_graph(m);
    return GB_OK;
}
extern "C" int gb_model_set_norms(gb_model* m, int layer, const float* a, const float* f) {
    if (!m || layer < 0 || layer >= m->c.n_layers || !a || !f) return GB_EINVAL;
    m->ra[layer] = a;
    m->rf[layer] = f;
    invalidate_graph(m);
    return GB_OK;
}
extern "C" int gb_model_set_head(gb_model* m, int emb_dtype, const void* emb, const float* rms_final, int lm_dtype,
                                 const void* lm) {
    if (!m || !emb || !rms_final || !lm) return GB_EINVAL;
    if (emb_dtype != GB_DT_Q4_K && emb_dtype != GB_DT_Q8_0 && emb_dtype != GB_DT_F32) return GB_EINVAL;
    MvPlan p;
    const int rc = mv_plan(&p, lm_dtype, lm, m->vocab_l, m->c.hidden_dim);   // this rank's vocabulary rows
    if (rc) return rc;
    m->emb = emb; m->emb_dt = emb_dtype; m->rms_final = rms_final; m->lm = lm; m->lm_dt = lm_dtype;
    m->lm_plan = p;
    invalidate_graph(m);
    return GB_OK;
}

extern "C" float* gb_model_k_cache(gb_model* m, int layer) {
    return (m && layer >= 0 && layer < m->c.n_layers) ? m->kc + (size_t)layer * m->kv_dim * m->c.max_seq : nullptr;
}
extern "C" float* gb_model_v_cache(gb_model* m, int layer) {
    return (m && layer >= 0 && layer < m->c.n_layers) ? m->vc + (size_t)layer * m->kv_dim * m->c.max_seq : nullptr;
}

// This rank's matrix shape per slot (rows, cols): q / k / v rows of its
// heads, wo columns of its heads, gate / up rows and ffn_down columns of its
// FFN slice (a Q6_K ffn_down shard is stored with rows padded to 8 blocks).
static void mat_shape(const gb_model* m, int which, int dtype, int* rows, int* cols) {
    const int H = m->c.hidden_dim, QD = m->nh * m->c.head_dim;
    switch (which) {
        case GB_WQ: *rows = QD; *cols = H; break;
        case GB_WK: case GB_WV: *rows = m->kv_dim; *cols = H; break;
        case GB_WO: *rows = H; *cols = QD; break;
        case GB_WGATE: case GB_WUP: *rows = m->ff; *cols = H; break;
        default: *rows = H; *cols = (dtype == GB_DT_Q6_K && (m->world > 1 || m->pad_down)) ? m->ff_pad : m->ff; break;
    }
}

// The slice of the full synthetic matrix `which` (stream stream_id) this rank
// holds, with the bytes the one-GPU model would have at those positions.
static int synth_slice(gb_model* m, int which, int dtype, void* p, uint64_t seed, uint64_t stream_id) {
    const gb_model_config& c = m->c;
    const int H = c.hidden_dim, hd = c.head_dim;
    const uint64_t nbH = H / 256;
    int rows, cols;
    mat_shape(m, which, dtype, &rows, &cols);
    switch (which) {
        case GB_WQ:
            return synth_blocks_shard(dtype, p, rows, nbH, nbH, (uint64_t)m->rank * rows, nbH, 0, seed, stream_id, m->stream);
        case GB_WK: case GB_WV:
            return synth_blocks_shard(dtype, p, rows, nbH, nbH, (uint64_t)m->rank * rows, nbH, 0, seed, stream_id, m->stream);
        case GB_WGATE: case GB_WUP:
            return synth_blocks_shard(dtype, p, rows, nbH, nbH, (uint64_t)m->rank * rows, nbH, 0, seed, stream_id, m->stream);
        case GB_WO: {
            const uint64_t sn = (uint64_t)m->nh * hd / 256;
            return synth_blocks_shard(dtype, p, rows, sn, sn, 0, (uint64_t)c.n_heads * hd / 256, m->rank * sn, seed,
                                      stream_id, m->stream);
        }
        default: {   // ffn_down: this rank's FFN columns, zero padding after them
            const uint64_t sn = (uint64_t)m->ff / 256, ldo = (uint64_t)cols / 256;
            if (ldo > sn &&
                cudaMemsetAsync(p, 0, (size_t)rows * ldo * gb_block_bytes(dtype), m->stream) != cudaSuccess)
                return GB_ECUDA;
            return synth_blocks_shard(dtype, p, rows, sn, ldo, 0, (uint64_t)c.ff_dim / 256, m->rank * sn, seed,
                                      stream_id, m->stream);
        }
    }
}

extern "C" int gb_model_synthesize(gb_model* m, uint64_t seed) {
    if (!m) return GB_EINVAL;
    const gb_model_config& c = m->c;
    const int H = c.hidden_dim;
    float* ones = (float*)dalloc(m, (size_t)H * 4);
    if (!ones) return GB_ENOMEM;
    int rc = gb_fill_f32(ones, H, 1.0f, m->stream);
    if (rc) return rc;
    // the synthesised Q6_K ffn_down rows are padded to 8-block multiples (the
    // tensor-map path); gb_model_set_matrix afterwards takes unpadded rows
    struct PadScope {
        gb_model* m;
        ~PadScope() { m->pad_down = false; }
    } pad_scope{m};
    m->pad_down = true;
    for (int l = 0; l < c.n_layers; l++) {
        for (int wi = 0; wi < GB_NMAT; wi++) {
            const int dtype = (wi == GB_WV || wi == GB_WDOWN) ? GB_DT_Q6_K : GB_DT_Q4_K;
            int rows, cols;
            mat_shape(m, wi, dtype, &rows, &cols);
            if (cols % 256) return GB_ESHAPE;
            const size_t nblk = (size_t)rows * (cols / 256);
            void* p = dalloc(m, nblk * gb_block_bytes(dtype) + 16);
            if (!p) return GB_ENOMEM;
            if ((rc = synth_slice(m, wi, dtype, p, seed, (uint64_t)(l * GB_NMAT + wi + 1)))) return rc;
            if ((rc = gb_model_set_matrix(m, l, wi, dtype, p))) return rc;
        }
        gb_model_set_norms(m, l, ones, ones);
    }
    const size_t eblk = (size_t)c.vocab_size * (H / 256);
    const size_t lblk = (size_t)m->vocab_l * (H / 256);
    void* e = dalloc(m, eblk * GB_Q4K_BYTES);
    void* lmp = dalloc(m, lblk * GB_Q6K_BYTES + 16);
    if (!e || !lmp) return GB_ENOMEM;
    if ((rc = gb_synth_blocks(GB_DT_Q4_K, e, eblk, seed, 1000001ull, m->stream))) return rc;   // every rank: full table
    if ((rc = synth_blocks_shard(GB_DT_Q6_K, lmp, m->vocab_l, H / 256, H / 256, (uint64_t)m->vocab_off, H / 256, 0,
                                 seed, 1000002ull, m->stream)))
        return rc;
    if ((rc = gb_model_set_head(m, GB_DT_Q4_K, e, ones, GB_DT_Q6_K, lmp))) return rc;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? GB_OK : GB_ECUDA;
}

namespace gb {
// One decode layer (engine.c:353-554) on stream st; shared by the model and
// the drop-in cuda_transformer_layer_gpu.
// Tensor parallelism with the hidden-state exchanges inside the matvecs:
// every matvec of the layer (and the output head) on the TMA path, and x
// small enough for the one-pass RMSNorm quantiser.
bool tp_fusable(const MvPlan* const* mv, int H) {
    if (H % 4 || H > 8192) return false;
    for (int i = 0; i < GB_NMAT; i++)
        if (mv[i]->kind != MV_TMA) return false;
    return true;
}

int enqueue_layer(const LayerArgs& a, cudaStream_t st) {
    const int H = a.H, F = a.ff;
    int rc;
    const bool tp = a.tp && a.tp->world > 1;
    const bool fx = tp && a.tp_fused;   // exchanges inside the matvecs
    const int c_wo = 2 * a.layer, c_dn = 2 * a.layer + 1;   // this layer's exchanges
    // hidden state read by the q/k/v and the gate/up matvecs.  One GPU: one
    // buffer updated in place by the residual adds.  Tensor parallel:
    // exchange c reads h[c & 1] and writes h[(c + 1) & 1]; with the exchanges
    // inside the matvecs the q/k/v matvec sums the previous layer's ffn_down
    // exchange (none before layer 0) and the gate/up matvec the wo exchange.
    float* hq = a.hidden;
    float* hf = a.hidden;
    if (tp) {
        hq = fx && a.layer > 0 ? a.tp->h[1] : a.tp->h[0];
        hf = fx ? a.tp->h[0] : a.tp->h[1];
    }
    MvTp tq, twp, tg, tdp;   // q/k/v input, wo push, gate/up input, ffn_down push
    if (fx) {
        tq = twp = tg = tdp = a.tp->mv();
        tq.H = twp.H = tg.H = tdp.H = H;
        if (a.layer > 0) {
            tq.in_call = c_wo - 1;
            tq.h_out = a.tp->h[0];
        }
        twp.push_call = c_wo;
        tg.in_call = c_wo;
        tg.h_out = a.tp->h[1];
        tdp.push_call = c_dn;
    }
    auto mv = [&](int which, const float* x, float* y, const float* res, const MvXform* xf,
                  const MvTp* tpx = nullptr) {
        return mv_launch(*a.mv[which], x, y, res, a.mv_ws, st, true, xf, tpx);
    };
    auto tma = [&](int which) { return a.mv[which]->kind == MV_TMA; };
    // RMSNorm and the SwiGLU product run inside the consuming matvecs' x
    // quantiser when those are on the TMA path (no separate launches)
    MvXform att, ffn, swi;
    att.mode = ffn.mode = MV_X_RMSNORM;
    att.w = a.ra;
    ffn.w = a.rf;
    att.eps = ffn.eps = a.eps;
    swi.mode = MV_X_SILU_MUL;
    swi.x2 = a.up;
    // matrices that share x and a format run as one launch
    auto group = [&](const int* which, int n, const float* x, float* const* ys, const MvXform* xf,
                     const MvTp* tpx) {
        const MvPlan* ps[3];
        for (int i = 0; i < n; i++) ps[i] = a.mv[which[i]];
        return mv_launch_group(ps, n, x, ys, nullptr, a.mv_ws, st, true, xf, tpx);
    };
    const MvTp* tqp = fx ? &tq : nullptr;
    if (tma(GB_WQ) && tma(GB_WK) && tma(GB_WV)) {
        const int qkv[3] = {GB_WQ, GB_WK, GB_WV};
        float* ys[3] = {a.q, a.k, a.v};
        const MvPlan* ps[3] = {a.mv[GB_WQ], a.mv[GB_WK], a.mv[GB_WV]};
        if (mv_groupable(ps, 3)) {
            if ((rc = group(qkv, 3, hq, ys, &att, tqp))) return rc;
        } else if (mv_groupable(ps, 2)) {
            if ((rc = group(qkv, 2, hq, ys, &att, tqp))) return rc;
            if ((rc = mv(GB_WV, hq, a.v, nullptr, &att, tqp))) return rc;
        } else {
            if ((rc = mv(GB_WQ, hq, a.q, nullptr, &att, tqp))) return rc;
            if ((rc = mv(GB_WK, hq, a.k, nullptr, &att, tqp))) return rc;
            if ((rc = mv(GB_WV, hq, a.v, nullptr, &att, tqp))) return rc;
        }
    } else {
        if ((rc = gb_rmsnorm(hq, a.ra, a.xn, H, a.eps, st))) return rc;
        if ((rc = mv(GB_WQ, a.xn, a.q, nullptr, nullptr))) return rc;
        if ((rc = mv(GB_WK, a.xn, a.k, nullptr, nullptr))) return rc;
        if ((rc = mv(GB_WV, a.xn, a.v, nullptr, nullptr))) return rc;
    }
    // wo's x arrives quantised from the attention launch: the CTA that
    // finishes a KV head quantises its 32-column groups of the output
    const bool aq = a.aq && tma(GB_WO) && a.mv[GB_WO]->cols == a.n_heads * a.hd;
    if ((rc = attention_decode_xq(a.q, a.k, a.v, a.kc, a.vc, a.rope, a.d_pos, a.n_heads, a.n_kv, a.hd, a.max_seq,
                                  a.attn, a.attn_ws, aq ? a.aq : nullptr, st, true)))
        return rc;
    MvXform woq;
    woq.mode = MV_X_PREQ;
    woq.xq = a.aq;
    const MvXform* wxf = aq ? &woq : nullptr;
    if (fx) {   // this rank's columns of wo, pushed to every rank
        if ((rc = mv(GB_WO, a.attn, a.tp->part, nullptr, wxf, &twp))) return rc;
    } else if (tp) {   // this rank's columns of wo, then the exchange as its own launch
        if ((rc = mv(GB_WO, a.attn, a.tp->part, nullptr, wxf))) return rc;
        if ((rc = tp_allreduce(*a.tp, a.tp->h[0], a.tp->h[1], H, c_wo, st))) return rc;
    } else if ((rc = mv(GB_WO, a.attn, a.hidden, a.hidden, wxf))) {
        return rc;
    }
    const MvTp* tgp = fx ? &tg : nullptr;
    // the gate / up launch also writes ffn_down's x quantised (one launch,
    // one format, one item per 32-row group, ffn_down on the TMA path)
    const MvPlan* pg = a.mv[GB_WGATE];
    const MvPlan* pu = a.mv[GB_WUP];
    const MvPlan* pd = a.mv[GB_WDOWN];
    const bool swq = a.swq && a.swq_tk && tma(GB_WGATE) && tma(GB_WUP) && tma(GB_WDOWN) && pg->dtype == pu->dtype &&
                     pg->nch == 1 && pu->nch == 1 && pg->rows == pu->rows && pd->cols % 256 == 0 &&
                     pd->cols >= pg->rows;
    if (tma(GB_WGATE) && tma(GB_WUP)) {
        const int gu[2] = {GB_WGATE, GB_WUP};
        float* ys[2] = {a.gate, a.up};
        const MvPlan* ps[2] = {a.mv[GB_WGATE], a.mv[GB_WUP]};
        if (mv_groupable(ps, 2)) {
            MvXform fq = ffn;
            if (swq) {
                fq.swq_out = a.swq;
                fq.swq_tk = a.swq_tk;
                fq.swq_K = pd->cols;
            }
            if ((rc = group(gu, 2, hf, ys, &fq, tgp))) return rc;
        } else {
            if ((rc = mv(GB_WGATE, hf, a.gate, nullptr, &ffn, tgp))) return rc;
            if ((rc = mv(GB_WUP, hf, a.up, nullptr, &ffn, tgp))) return rc;
        }
    } else {
        if ((rc = gb_rmsnorm(hf, a.rf, a.xn, H, a.eps, st))) return rc;
        if ((rc = mv(GB_WGATE, a.xn, a.gate, nullptr, nullptr))) return rc;
        if ((rc = mv(GB_WUP, a.xn, a.up, nullptr, nullptr))) return rc;
    }
    float* dy = tp ? a.tp->part : a.hidden;
    const float* dres = tp ? nullptr : a.hidden;
    const bool gu_grouped = [&] {
        const MvPlan* ps[2] = {pg, pu};
        return tma(GB_WGATE) && tma(GB_WUP) && mv_groupable(ps, 2);
    }();
    if (swq && gu_grouped) {   // x arrives quantised from the gate / up launch
        MvXform pq;
        pq.mode = MV_X_PREQ;
        pq.xq = a.swq;
        rc = mv(GB_WDOWN, a.gate, dy, dres, &pq, fx ? &tdp : nullptr);
    } else if (tma(GB_WDOWN)) {
        rc = mv(GB_WDOWN, a.gate, dy, dres, &swi, fx ? &tdp : nullptr);
    } else {
        if ((rc = gb_silu_mul(a.gate, a.up, F, st))) return rc;
        rc = mv(GB_WDOWN, a.gate, dy, dres, nullptr);
    }
    if (rc || !tp || fx) return rc;
    return tp_allreduce(*a.tp, a.tp->h[1], a.tp->h[0], H, c_dn, st);
}

size_t layer_ws_bytes(const MvPlan* const* mv) {
    size_t need = 0;
    for (int i = 0; i < GB_NMAT; i++) need = std::max(need, mv_ws_bytes(*mv[i]));
    const MvPlan* qkv[3] = {mv[GB_WQ], mv[GB_WK], mv[GB_WV]};
    const MvPlan* gu[2] = {mv[GB_WGATE], mv[GB_WUP]};
    need = std::max(need, mv_ws_bytes_group(qkv, 3));
    need = std::max(need, mv_ws_bytes_group(qkv, 2));
    need = std::max(need, mv_ws_bytes_group(gu, 2));
    return need;
}

int embed(const void* emb, int dtype, const int* d_token, int vocab, int H, float* out, unsigned* err, cudaStream_t st,
          unsigned long long* step, int rows) {
    k_embed<<<dim3((H + 255) / 256, rows), 256, 0, st>>>(emb, dtype, d_token, vocab, H, out, err, step);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
int rmsnorm_rows(const float* x, const float* w, float* out, int n, int rows, float eps, cudaStream_t st) {
    k_rmsnorm<<<rows, 1024, 0, st>>>(x, w, out, n, eps);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
int tp_allreduce(const TpCtx& tp, const float* h_in, float* h_out, int H, int call, cudaStream_t st) {
    k_tp_allreduce<<<tp.world, 512, 0, st>>>(tp.part, h_in, h_out, H, tp.rank, tp.world, tp.d_peers, tp.d_step,
                                             tp.calls, call, tp.err);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
int set_device_int(int* p, int v, cudaStream_t st) {
    k_set_int<<<1, 1, 0, st>>>(p, v);
    return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
}
}  // namespace gb

// Tensor parallel with the exchanges inside the matvecs: every layer and the
// output head on the TMA path (otherwise each exchange is its own launch).
static bool tp_fused(const gb_model* m) {
    const char* e = getenv("GB_TP_FUSED");   // 0: every exchange as its own launch
    if (e && e[0] == '0') return false;
    if (m->lm_plan.kind != MV_TMA) return false;
    for (int l = 0; l < m->c.n_layers; l++) {
        const MvPlan* mv[GB_NMAT];
        for (int i = 0; i < GB_NMAT; i++) mv[i] = &m->plan[(size_t)l * GB_NMAT + i];
        if (!tp_fusable(mv, m->c.hidden_dim)) return false;
    }
    return true;
}

// Enqueue one decode step on stream st.
static int enqueue_argmax(gb_model* m, const float* lg, int* d_next, cudaStream_t st);
static int enqueue_head(gb_model* m, const float* hx, float* lg, bool fx, cudaStream_t st);
static int enqueue_step(gb_model* m, const int* d_token, const int* d_pos, float* d_logits, int* d_next,
                        cudaStream_t st) {
    const gb_model_config& c = m->c;
    const int H = c.hidden_dim;
    int rc;
    if ((rc = embed(m->emb, m->emb_dt, d_token, c.vocab_size, H, m->hidden, m->err, st, m->d_step))) return rc;
    const bool fx = m->world > 1 && tp_fused(m);
    for (int l = 0; l < c.n_layers; l++) {
        LayerArgs a;
        a.tp = m->world > 1 ? &m->tp : nullptr;
        a.tp_fused = fx;
        a.swq = m->swq;
        a.swq_tk = m->swq_tk;
        a.aq = m->world == 1 ? m->aq : nullptr;   // one GPU only (the tensor-parallel wo keeps its own quantiser)
        a.layer = l;
        for (int i = 0; i < GB_NMAT; i++) a.mv[i] = &m->plan[(size_t)l * GB_NMAT + i];
        a.mv_ws = m->mv_ws;
        a.ra = m->ra[l]; a.rf = m->rf[l];
        a.kc = gb_model_k_cache(m, l); a.vc = gb_model_v_cache(m, l);
        a.rope = m->rope; a.d_pos = d_pos; a.attn_ws = m->attn_ws;
        a.hidden = m->hidden; a.xn = m->xn; a.q = m->q; a.k = m->k; a.v = m->v; a.attn = m->attn;
        a.gate = m->gate; a.up = m->up;
        a.H = H; a.n_heads = m->nh; a.n_kv = m->nkv; a.hd = c.head_dim; a.ff = m->ff;
        a.max_seq = c.max_seq; a.eps = c.rms_eps;
        if ((rc = enqueue_layer(a, st))) return rc;
    }
    float* lg = d_logits ? d_logits : m->logits;
    if ((rc = enqueue_head(m, fx ? m->tp.h[1] : m->hidden, lg, fx, st))) return rc;
    return enqueue_argmax(m, lg, d_next, st);
}

// Final RMSNorm and the output head of hidden row hx (engine.c:580-592).
static int enqueue_head(gb_model* m, const float* hx, float* lg, bool fx, cudaStream_t st) {
    const gb_model_config& c = m->c;
    const int H = c.hidden_dim;
    int rc;
    if (m->lm_plan.kind == MV_TMA) {   // final RMSNorm inside the output-head matvec
        MvXform fin;
        fin.mode = MV_X_RMSNORM;
        fin.w = m->rms_final;
        fin.eps = c.rms_eps;
        MvTp th;   // tensor parallel: the head sums the last layer's ffn_down exchange
        if (fx) {
            th = m->tp.mv();
            th.H = H;
            th.in_call = 2 * c.n_layers - 1;
            th.h_out = m->tp.h[0];
        }
        return mv_launch(m->lm_plan, hx, lg, nullptr, m->mv_ws, st, true, &fin, fx ? &th : nullptr);
    }
    if ((rc = gb_rmsnorm(hx, m->rms_final, m->xn, H, c.rms_eps, st))) return rc;
    return mv_launch(m->lm_plan, m->xn, lg, nullptr, m->mv_ws, st, true);
}

// Next token = first index of the largest logit (over the ranks' slices).
static int enqueue_argmax(gb_model* m, const float* lg, int* d_next, cudaStream_t st) {
    const gb_model_config& c = m->c;
    const int H = c.hidden_dim;
    const int G = std::min(AM_MAX_CTAS, (m->vocab_l + 4095) / 4096);
    ArgPart* part = static_cast<ArgPart*>(m->am_ws);
    k_argmax_split<<<G, 1024, 0, st>>>(lg, m->vocab_l, d_next, part, reinterpret_cast<unsigned*>(part + AM_MAX_CTAS),
                                       m->world > 1 ? m->am_res : nullptr, m->vocab_off);
    if (cudaGetLastError() != cudaSuccess) return GB_ECUDA;
    if (m->world > 1) {   // the best (value, index) over the ranks' vocabulary slices
        k_tp_argmax<<<1, 32, 0, st>>>(m->am_res, d_next, H, m->rank, m->world, m->d_peers, m->d_step, m->tp.calls,
                                      2 * c.n_layers, m->err);
        if (cudaGetLastError() != cudaSuccess) return GB_ECUDA;
    }
    return GB_OK;
}

// All weights set, and the shared matvec workspace sized for every plan.
static bool model_ready(gb_model* m) {
    if (m->world > 1 && !m->comm_ready) return false;   // gb_model_comm_open first
    for (size_t i = 0; i < m->w.size(); i++) if (!m->w[i]) return false;
    for (int l = 0; l < m->c.n_layers; l++) if (!m->ra[l] || !m->rf[l]) return false;
    if (!(m->emb && m->lm && m->rms_final)) return false;
    size_t need = mv_ws_bytes(m->lm_plan);
    for (int l = 0; l < m->c.n_layers; l++) {
        const MvPlan* mv[GB_NMAT];
        for (int i = 0; i < GB_NMAT; i++) mv[i] = &m->plan[(size_t)l * GB_NMAT + i];
        need = std::max(need, layer_ws_bytes(mv));
    }
    if (need > m->mv_ws_size) {
        void* p = dalloc(m, need);
        if (!p || cudaMemsetAsync(p, 0, need, m->stream) != cudaSuccess ||
            cudaStreamSynchronize(m->stream) != cudaSuccess)
            return false;
        m->mv_ws = p;
        m->mv_ws_size = need;
        invalidate_graph(m);
    }
    return true;
}

extern "C" int gb_model_decode(gb_model* m, const int* d_token, const int* d_pos, float* d_logits, int* d_next,
                               void* stream) {
    if (!m || !d_token || !d_pos || !d_next) return GB_EINVAL;
    if (!model_ready(m)) return GB_EINVAL;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
    const void* key[5] = {d_token, d_pos, d_logits, d_next, st};
    if (!m->exec || memcmp(key, m->key, sizeof(key)) != 0) {
        invalidate_graph(m);
        cudaStream_t cap = m->stream;   // capture on the model's own stream, replay on st
        if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed) != cudaSuccess) return GB_ECUDA;
        const int rc = enqueue_step(m, d_token, d_pos, d_logits, d_next, cap);
        cudaGraph_t g = nullptr;
        const cudaError_t ec = cudaStreamEndCapture(cap, &g);
        if (rc != GB_OK || ec != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return rc != GB_OK ? rc : GB_ECUDA;
        }
        const cudaError_t ei = cudaGraphInstantiate(&m->exec, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) { m->exec = nullptr; return GB_ECUDA; }
        memcpy(m->key, key, sizeof(key));
    }
    return cudaGraphLaunch(m->exec, st) == cudaSuccess ? GB_OK : GB_ECUDA;
}

// Capture the sequence [enqueue] on the model stream into a graph.
template <class Fn>
static int capture(gb_model* m, cudaGraphExec_t* exec, Fn&& enqueue) {
    cudaStream_t cap = m->stream;
    if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed) != cudaSuccess) return GB_ECUDA;
    const int rc = enqueue(cap);
    cudaGraph_t g = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(cap, &g);
    if (rc != GB_OK || ec != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return rc != GB_OK ? rc : GB_ECUDA;
    }
    const cudaError_t ei = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) { *exec = nullptr; return GB_ECUDA; }
    return GB_OK;
}

extern "C" int gb_model_generate(gb_model* m, int* d_token, int* d_pos, int n_steps, int* d_tokens_out,
                                 void* stream) {
    if (!m || !d_token || !d_pos || n_steps < 0) return GB_EINVAL;
    if (!model_ready(m)) return GB_EINVAL;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
    const void* key[4] = {d_token, d_pos, d_tokens_out, st};
    if (!m->gen_exec || memcmp(key, m->gen_key, sizeof(key)) != 0) {
        if (m->gen_exec) { cudaGraphExecDestroy(m->gen_exec); m->gen_exec = nullptr; }
        int* cnt = m->d_count;
        int* nxt = m->d_next;
        const int rc = capture(m, &m->gen_exec, [&](cudaStream_t cap) {
            int r = enqueue_step(m, d_token, d_pos, m->logits, nxt, cap);
            if (r) return r;
            k_advance<<<1, 1, 0, cap>>>(d_token, nxt, d_pos, d_tokens_out, cnt);
            return cudaGetLastError() == cudaSuccess ? GB_OK : GB_ECUDA;
        });
        if (rc) return rc;
        memcpy(m->gen_key, key, sizeof(key));
    }
    GB_CUDA_TRY(cudaMemsetAsync(m->d_count, 0, sizeof(int), st));
    for (int i = 0; i < n_steps; i++) GB_CUDA_TRY(cudaGraphLaunch(m->gen_exec, st));
    return GB_OK;
}

extern "C" int gb_model_error(gb_model* m) {
    if (!m) return GB_EINVAL;
    unsigned herr = 0;
    GB_CUDA_TRY(cudaStreamSynchronize(m->stream));
    GB_CUDA_TRY(cudaMemcpy(&herr, m->err, sizeof(unsigned), cudaMemcpyDeviceToHost));
    return -(int)herr;
}

extern "C" int gb_model_fill_kv(gb_model* m, int n_pos, uint64_t seed) {
    if (!m || n_pos < 0 || n_pos > m->c.max_seq) return GB_EINVAL;
    const gb_model_config& c = m->c;
    for (int l = 0; l < c.n_layers; l++)
        for (int which = 0; which < 2; which++) {
            float* base = which ? gb_model_v_cache(m, l) : gb_model_k_cache(m, l);
            for (int h = 0; h < m->nkv; h++) {   // this rank's KV heads, numbered globally
                float* p = base + (size_t)h * c.max_seq * c.head_dim;
                const int hg = m->rank * m->nkv + h;
                const int rc = gb_synth_normal(p, (size_t)n_pos * c.head_dim, seed,
                                               (uint64_t)((l * 2 + which) * 256 + hg) + 5000000ull, m->stream);
                if (rc) return rc;
            }
        }
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? GB_OK : GB_ECUDA;
}

extern "C" int gb_model_launches_per_step(const gb_model* m) {
    // embed + per layer (7 matvecs, attention, and the RMSNorm / SwiGLU
    // kernels that are not fused into a TMA matvec) + output head (+ final
    // norm when not fused) + argmax
    if (!m) return 0;
    int n = 1;
    for (int l = 0; l < m->c.n_layers; l++) {
        auto P = [&](int w) { return &m->plan[(size_t)l * GB_NMAT + w]; };
        auto tma = [&](int w) { return P(w)->kind == MV_TMA; };
        const MvPlan* qkv[3] = {P(GB_WQ), P(GB_WK), P(GB_WV)};
        const MvPlan* gu[2] = {P(GB_WGATE), P(GB_WUP)};
        n += 1 + 1 + 1;   // attention, wo, ffn_down
        if (tma(GB_WQ) && tma(GB_WK) && tma(GB_WV))
            n += mv_groupable(qkv, 3) ? 1 : (mv_groupable(qkv, 2) ? 2 : 3);
        else
            n += 4;   // RMSNorm + three matvecs
        if (tma(GB_WGATE) && tma(GB_WUP))
            n += mv_groupable(gu, 2) ? 1 : 2;
        else
            n += 3;
        n += tma(GB_WDOWN) ? 0 : 1;
    }
    n += m->lm_plan.kind == MV_TMA ? 1 : 2;
    if (m->world > 1)   // all-reduces after wo / ffn_down (unless inside the matvecs), argmax merge
        n += (tp_fused(m) ? 0 : 2 * m->c.n_layers) + 1;
    return n + 1;
}

extern "C" int gb_model_decode_host(gb_model* m, int token, int pos, int* h_next, float* h_logits) {
    if (!m || !h_next) return GB_EINVAL;
    if (pos < 0 || pos >= m->c.max_seq) return GB_EPOS;
    if (token < 0 || token >= m->c.vocab_size) return GB_EINVAL;
    cudaStream_t st = m->stream;
    m->h_io[0] = token;
    m->h_io[1] = pos;
    GB_CUDA_TRY(cudaMemcpyAsync(m->d_tok, &m->h_io[0], 2 * sizeof(int), cudaMemcpyHostToDevice, st));   // token, pos
    int rc = gb_model_decode(m, m->d_tok, m->d_pos, m->logits, m->d_next, st);
    if (rc) return rc;
    GB_CUDA_TRY(cudaMemcpyAsync(&m->h_io[2], m->d_next, 2 * sizeof(int), cudaMemcpyDeviceToHost, st));   // next, error
    if (h_logits)
        GB_CUDA_TRY(cudaMemcpyAsync(h_logits, m->logits, (size_t)m->vocab_l * 4, cudaMemcpyDeviceToHost, st));
    GB_CUDA_TRY(cudaStreamSynchronize(st));
    const unsigned herr = static_cast<unsigned>(m->h_io[3]);
    if (herr) return -(int)herr;
    *h_next = m->h_io[2];
    return GB_OK;
}

// ---------------------------------------------------------------- prefill
// Prompt tokens per pass through the layers (GB_PREFILL_CHUNK overrides): a
// longer prompt runs as consecutive chunks, each attending to the cache the
// earlier ones filled.
static int prefill_chunk() {
    const char* e = getenv("GB_PREFILL_CHUNK");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 4096;
}

// Activation floats per prompt token: hidden, xn, q, k, v, attn, gate, up
// (gate / up rows ff_pad wide: ffn_down's columns, zero past the FFN), and
// the current GEMM input's token scales; its split (pf_split_floats) follows.
static size_t pf_split_k(const gb_model* m) {
    return std::max({(size_t)m->c.hidden_dim, (size_t)m->nh * m->c.head_dim, (size_t)m->ff_pad});
}
static size_t pf_floats_per_token(const gb_model* m) {
    const int H = m->c.hidden_dim, QD = m->nh * m->c.head_dim;
    return 2 * (size_t)H + 2 * (size_t)QD + 2 * (size_t)m->kv_dim + 2 * (size_t)m->ff_pad + 1;
}
// The split of the current GEMM input for cap prompt rows, in floats: hi and
// lo halves of up to pf_split_k columns over the padded rows.
static size_t pf_split_floats(const gb_model* m, int cap) {
    return (size_t)gemm_split_rows(cap) * pf_split_k(m);
}
// Where the split starts: after the per-token floats, 256-byte aligned.
static size_t pf_split_offset(const gb_model* m, int cap) {
    return ((size_t)cap * pf_floats_per_token(m) + 63) / 64 * 64;
}

static int pf_reserve(gb_model* m, int T) {
    if (!m->pf_side) {   // the side stream and its events (created once)
        if (cudaStreamCreateWithFlags(&m->pf_side, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&m->pf_fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&m->pf_join, cudaEventDisableTiming) != cudaSuccess)
            return GB_ECUDA;
    }
    if (T <= m->pf_cap) return GB_OK;
    if (m->pf) {   // earlier prefills on this stream may still read it
        GB_CUDA_TRY(cudaStreamSynchronize(m->stream));
        GB_CUDA_TRY(cudaDeviceSynchronize());
        cudaFree(m->pf);
        m->pf = nullptr;
        m->pf_cap = 0;
    }
    const size_t bytes = (pf_split_offset(m, T) + pf_split_floats(m, T)) * sizeof(float);
    if (cudaMalloc(&m->pf, bytes) != cudaSuccess) {
        m->pf = nullptr;
        return GB_ENOMEM;
    }
    // zero once: the gate / up columns past the FFN stay zero (never written)
    if (cudaMemsetAsync(m->pf, 0, bytes, m->stream) != cudaSuccess || cudaStreamSynchronize(m->stream) != cudaSuccess)
        return GB_ECUDA;
    m->pf_cap = T;
    return GB_OK;
}

extern "C" int gb_model_prefill(gb_model* m, const int* d_tokens, int n_tokens, int pos, float* d_logits, int* d_next,
                                void* stream) {
    if (!m || !d_tokens || !d_next || n_tokens <= 0) return GB_EINVAL;
    const gb_model_config& c = m->c;
    if (pos < 0 || (long long)pos + n_tokens > c.max_seq) return GB_EPOS;
    if (m->world != 1) return GB_EINVAL;   // one GPU: the matrices are whole
    if (!model_ready(m)) return GB_EINVAL;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
    const int chunk = std::min(n_tokens, prefill_chunk());
    int rc;
    if ((rc = pf_reserve(m, chunk))) return rc;
    const int H = c.hidden_dim, QD = m->nh * c.head_dim, KVD = m->kv_dim, F = m->ff;
    float* base = static_cast<float*>(m->pf);
    const size_t cap = (size_t)m->pf_cap;
    PrefillArgs a;
    a.hidden = base;
    a.xn = a.hidden + cap * H;
    a.q = a.xn + cap * H;
    a.attn = a.q + cap * QD;
    a.k = a.attn + cap * QD;
    a.v = a.k + cap * KVD;
    a.gate = a.v + cap * KVD;
    a.up = a.gate + cap * (size_t)m->ff_pad;
    a.xinv = a.up + cap * (size_t)m->ff_pad;
    a.xh = base + pf_split_offset(m, (int)cap);
    a.xl = static_cast<float*>(a.xh) + pf_split_floats(m, (int)cap) / 2;
    a.err = m->err;
    a.side = m->pf_side;
    a.fork = m->pf_fork;
    a.join = m->pf_join;
    a.rope = m->rope;
    a.H = H; a.n_heads = m->nh; a.n_kv = m->nkv; a.hd = c.head_dim; a.ff = F; a.max_seq = c.max_seq;
    a.eps = c.rms_eps;
    int T = 0;
    for (int c0 = 0; c0 < n_tokens; c0 += chunk) {
        T = std::min(chunk, n_tokens - c0);
        if ((rc = embed(m->emb, m->emb_dt, d_tokens + c0, c.vocab_size, H, a.hidden, m->err, st, nullptr, T)))
            return rc;
        a.T = T;
        a.pos0 = pos + c0;
        for (int l = 0; l < c.n_layers; l++) {
            for (int i = 0; i < GB_NMAT; i++) {
                a.w[i] = m->w[(size_t)l * GB_NMAT + i];
                a.dt[i] = m->dt[(size_t)l * GB_NMAT + i];
            }
            a.ra = m->ra[l]; a.rf = m->rf[l];
            a.kc = gb_model_k_cache(m, l); a.vc = gb_model_v_cache(m, l);
            a.fk = m->plan[(size_t)l * GB_NMAT + GB_WDOWN].cols;   // ff, or ff_pad for padded rows
            if ((rc = enqueue_prefill_layer(a, st))) return rc;
        }
    }
    float* lg = d_logits ? d_logits : m->logits;
    if ((rc = enqueue_head(m, a.hidden + (size_t)(T - 1) * H, lg, false, st))) return rc;
    return enqueue_argmax(m, lg, d_next, st);
}

extern "C" int gb_model_prefill_host(gb_model* m, const int* h_tokens, int n_tokens, int pos, int* h_next,
                                     float* h_logits) {
    if (!m || !h_tokens || !h_next || n_tokens <= 0) return GB_EINVAL;
    cudaStream_t st = m->stream;
    if (n_tokens > m->pf_tok_cap) {
        GB_CUDA_TRY(cudaStreamSynchronize(st));
        if (m->pf_tok) cudaFree(m->pf_tok);
        m->pf_tok = nullptr;
        m->pf_tok_cap = 0;
        GB_CUDA_TRY(cudaMalloc(&m->pf_tok, (size_t)n_tokens * sizeof(int)));
        m->pf_tok_cap = n_tokens;
    }
    GB_CUDA_TRY(cudaMemcpyAsync(m->pf_tok, h_tokens, (size_t)n_tokens * sizeof(int), cudaMemcpyHostToDevice, st));
    int rc = gb_model_prefill(m, m->pf_tok, n_tokens, pos, m->logits, m->d_next, st);
    if (rc) return rc;
    GB_CUDA_TRY(cudaMemcpyAsync(&m->h_io[2], m->d_next, 2 * sizeof(int), cudaMemcpyDeviceToHost, st));   // next, error
    if (h_logits)
        GB_CUDA_TRY(cudaMemcpyAsync(h_logits, m->logits, (size_t)m->vocab_l * 4, cudaMemcpyDeviceToHost, st));
    GB_CUDA_TRY(cudaStreamSynchronize(st));
    const unsigned herr = static_cast<unsigned>(m->h_io[3]);
    if (herr) return -(int)herr;
    *h_next = m->h_io[2];
    return GB_OK;
}

extern "C" double gb_model_step_bytes(const gb_model* m, int pos) {
    if (!m) return 0.0;
    const gb_model_config& c = m->c;
    double b = 0.0;
    for (int l = 0; l < c.n_layers; l++)
        for (int wi = 0; wi < GB_NMAT; wi++) {
            int rows, cols;
            const int dt = m->dt[(size_t)l * GB_NMAT + wi];
            mat_shape(m, wi, dt, &rows, &cols);
            b += (double)gb_matrix_bytes(dt, rows, cols);
        }
    b += (double)gb_matrix_bytes(m->lm_dt, m->vocab_l, c.hidden_dim);
    b += (double)(2 * c.n_layers + 1) * c.hidden_dim * 4;                   // norm weights
    b += 2.0 * c.n_layers * m->kv_dim * (double)(pos + 1) * 4;              // K and V read
    b += 2.0 * c.n_layers * m->kv_dim * 4;                                  // append
    b += (double)gb_matrix_bytes(m->emb_dt == GB_DT_F32 ? GB_DT_Q4_K : m->emb_dt, 1, c.hidden_dim);
    return b;
}

