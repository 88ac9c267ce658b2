// gb_abi.cu -- the drop-in extern "C" symbols the unchanged Guanaco engine,
// loader and KV cache bind (see include/guanaco_b200.h for the reference
// interface each one replaces), plus the host-buffer matvec used by the
// backend vtable (gb_backend.c).
//
// State: one context per CUDA device (stream, activations, per-layer device
// KV caches sized from max_seq, RoPE table, attention workspace, device copies
// of norm weights keyed by host pointer, and device copies of weights that
// were never uploaded (e.g. lm_head, src/engine/loader.c:677-729 uploads only
// per-layer tensors) keyed by host pointer).  Calls are serialised by a mutex,
// as the engine drives them from one host thread (backend.h threading model).
#include "gb_common.cuh"
#include "gb_internal.h"

#include <algorithm>
#include <cstring>

#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <unordered_map>
#include <vector>

namespace gb {

struct LayerKV {
    float* k = nullptr;
    float* v = nullptr;
    int n_kv = 0, hd = 0, max_seq = 0;
    int valid = 0;   // positions [0, valid) mirror the host cache
};

struct Ctx {
    int dev = -1;
    cudaStream_t st = nullptr;
    // activations
    int H = 0, KV = 0, F = 0;
    float *hidden = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *gate = nullptr, *up = nullptr;
    int* d_pos = nullptr;
    // host-buffer matvec staging
    float *mx = nullptr, *my = nullptr;
    size_t mx_n = 0, my_n = 0;
    // attention state
    float* rope = nullptr;
    int rope_seq = 0, rope_hd = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int ws_shape[4] = {0, 0, 0, 0};   // (n_heads, n_kv, hd, max_seq) the ticket words were zeroed for
    std::vector<LayerKV> kv;
    struct CachedNorm {
        float* d = nullptr;
        std::vector<float> host;   // the uploaded values (a reused host address must match them)
    };
    std::unordered_map<const void*, CachedNorm> norm_cache;
    struct CachedWeight {
        void* d = nullptr;
        size_t bytes = 0;
        uint64_t sig = 0;        // checksum of sampled bytes (detects a reused host address)
        uint64_t last_use = 0;   // use clock at the last call (least recently used goes first)
    };
    std::unordered_map<const void*, CachedWeight> weight_cache;
    size_t weight_cache_bytes = 0;
    uint64_t use_clock = 0;
    // prepared matvecs keyed by device weight pointer, and their workspace
    std::unordered_map<const void*, MvPlan> plans;
    void* mv_ws = nullptr;
    size_t mv_ws_size = 0;
};

static std::mutex g_mu;
static Ctx g_ctx[16];

static Ctx* ctx() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return nullptr;
    Ctx* c = &g_ctx[dev];
    if (c->dev < 0) {
        if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        c->dev = dev;
    }
    return c;
}

static bool grow(float** p, size_t* cap, size_t n) {
    if (*cap >= n) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, n * sizeof(float)) != cudaSuccess) { *p = nullptr; return false; }
    *cap = n;
    return true;
}

static bool ensure_acts(Ctx* c, int H, int KV, int F) {
    if (c->H >= H && c->KV >= KV && c->F >= F && c->hidden) return true;
    float** bufs[] = {&c->hidden, &c->xn, &c->q, &c->k, &c->v, &c->attn, &c->gate, &c->up};
    for (float** b : bufs) if (*b) { cudaFree(*b); *b = nullptr; }
    const int XN = H > F ? H : F;
    const size_t n[] = {(size_t)H, (size_t)XN, (size_t)H, (size_t)KV, (size_t)KV, (size_t)H, (size_t)F, (size_t)F};
    for (int i = 0; i < 8; i++)
        if (cudaMalloc(bufs[i], n[i] * sizeof(float)) != cudaSuccess) { *bufs[i] = nullptr; c->H = 0; return false; }
    if (!c->d_pos && cudaMalloc(&c->d_pos, 16) != cudaSuccess) { c->d_pos = nullptr; return false; }
    c->H = H; c->KV = KV; c->F = F;
    return true;
}

static bool ensure_rope(Ctx* c, int max_seq, int hd) {
    if (c->rope && c->rope_seq >= max_seq && c->rope_hd == hd) return true;
    if (c->rope) cudaFree(c->rope);
    c->rope = nullptr;
    if (cudaMalloc(&c->rope, (size_t)max_seq * hd * sizeof(float)) != cudaSuccess) { c->rope = nullptr; return false; }
    // RoPE theta is hard-coded to 500000 by the reference (kernels_cpu.c:408).
    if (gb_rope_table(c->rope, max_seq, hd, 500000.0f, c->st) != GB_OK) return false;
    c->rope_seq = max_seq;
    c->rope_hd = hd;
    return true;
}

static bool ensure_ws(Ctx* c, int n_heads, int n_kv, int hd, int max_seq) {
    const size_t need = gb_attn_workspace_bytes(n_heads, n_kv, hd, max_seq);
    if (need == 0) return false;
    const int shape[4] = {n_heads, n_kv, hd, max_seq};
    const bool same = std::equal(shape, shape + 4, c->ws_shape);
    if (c->ws && c->ws_bytes >= need) {
        // the tickets sit after the partials, so another shape puts them on
        // words that held partials: zero again (in stream order) on a change
        if (same) return true;
    } else {
        if (c->ws) { cudaStreamSynchronize(c->st); cudaFree(c->ws); }
        c->ws = nullptr;
        c->ws_bytes = 0;
        if (cudaMalloc(&c->ws, need) != cudaSuccess) { c->ws = nullptr; return false; }
        c->ws_bytes = need;
    }
    // zeroed in stream order: the split-K tickets must read 0 on first use
    std::fill(c->ws_shape, c->ws_shape + 4, 0);
    if (cudaMemsetAsync(c->ws, 0, c->ws_bytes, c->st) != cudaSuccess) return false;
    std::copy(shape, shape + 4, c->ws_shape);
    return true;
}

// Device KV of one layer, created zeroed on first use.
static LayerKV* layer_kv(Ctx* c, int layer, int n_kv, int hd, int max_seq) {
    if (layer < 0 || layer > 4096) return nullptr;
    if ((int)c->kv.size() <= layer) c->kv.resize(layer + 1);
    LayerKV& L = c->kv[layer];
    if (L.k && L.n_kv == n_kv && L.hd == hd && L.max_seq == max_seq) return &L;
    if (L.k) { cudaFree(L.k); cudaFree(L.v); }
    L = LayerKV();
    const size_t bytes = (size_t)n_kv * max_seq * hd * sizeof(float);
    if (cudaMalloc(&L.k, bytes) != cudaSuccess) { L.k = nullptr; return nullptr; }
    if (cudaMalloc(&L.v, bytes) != cudaSuccess) { cudaFree(L.k); L.k = nullptr; L.v = nullptr; return nullptr; }
    cudaMemsetAsync(L.k, 0, bytes, c->st);
    cudaMemsetAsync(L.v, 0, bytes, c->st);
    L.n_kv = n_kv; L.hd = hd; L.max_seq = max_seq;
    return &L;
}

// Copy positions [p0, p1) of the host KV (head stride stride0 floats) into the
// device cache (head stride max_seq * hd).
static int upload_kv(Ctx* c, LayerKV* L, const float* hk, const float* hv, int stride0, int p0, int p1) {
    if (p1 <= p0) return GB_OK;
    const size_t w = (size_t)(p1 - p0) * L->hd * sizeof(float);
    const size_t dp = (size_t)L->max_seq * L->hd * sizeof(float), hp = (size_t)stride0 * sizeof(float);
    const size_t off_d = (size_t)p0 * L->hd, off_h = (size_t)p0 * L->hd;
    GB_CUDA_TRY(cudaMemcpy2DAsync(L->k + off_d, dp, hk + off_h, hp, w, L->n_kv, cudaMemcpyHostToDevice, c->st));
    GB_CUDA_TRY(cudaMemcpy2DAsync(L->v + off_d, dp, hv + off_h, hp, w, L->n_kv, cudaMemcpyHostToDevice, c->st));
    return GB_OK;
}

// Norm weights are small (H floats): a cached device copy is reused only when
// the host values are identical, so a host buffer freed and reallocated at
// the same address (or resized) is uploaded again.
static const float* cached_norm(Ctx* c, const float* h, int n) {
    const size_t bytes = (size_t)n * sizeof(float);
    Ctx::CachedNorm& e = c->norm_cache[h];
    if (e.d && e.host.size() == (size_t)n && memcmp(e.host.data(), h, bytes) == 0) return e.d;
    if (e.d) {   // kernels still queued may read the old copy
        cudaStreamSynchronize(c->st);
        cudaFree(e.d);
        e.d = nullptr;
    }
    e.host.assign(h, h + n);
    void* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess ||
        cudaMemcpyAsync(d, e.host.data(), bytes, cudaMemcpyHostToDevice, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess) {
        if (d) cudaFree(d);
        c->norm_cache.erase(h);
        return nullptr;
    }
    e.d = static_cast<float*>(d);
    return e.d;
}

// Upload `size` bytes through a pinned bounce buffer: the CPU reads the
// source pages itself, which is safe for mmap'd MAP_PRIVATE file pages.
static void* upload_bytes(const void* host, size_t size, cudaStream_t st) {
    void* d = nullptr;
    if (cudaMalloc(&d, size ? size : 1) != cudaSuccess) return nullptr;
    const size_t CH = (size_t)32 << 20;
    void* pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool ok = cudaMallocHost(&pin[0], CH) == cudaSuccess && cudaMallocHost(&pin[1], CH) == cudaSuccess &&
              cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming) == cudaSuccess;
    for (size_t off = 0, i = 0; ok && off < size; off += CH, i ^= 1) {
        const size_t n = size - off < CH ? size - off : CH;
        ok &= cudaEventSynchronize(ev[i]) == cudaSuccess;
        memcpy(pin[i], static_cast<const uint8_t*>(host) + off, n);
        ok &= cudaMemcpyAsync(static_cast<uint8_t*>(d) + off, pin[i], n, cudaMemcpyHostToDevice, st) == cudaSuccess;
        ok &= cudaEventRecord(ev[i], st) == cudaSuccess;
    }
    ok &= cudaStreamSynchronize(st) == cudaSuccess;
    for (int i = 0; i < 2; i++) {
        if (pin[i]) cudaFreeHost(pin[i]);
        if (ev[i]) cudaEventDestroy(ev[i]);
    }
    if (!ok) { cudaFree(d); return nullptr; }
    return d;
}

// y = W x with host x / y and a device W; synchronous.
static int matvec_hostio(Ctx* c, int dtype, const void* dW, int rows, int cols, const float* hx, float* hy) {
    if (!grow(&c->mx, &c->mx_n, (size_t)cols) || !grow(&c->my, &c->my_n, (size_t)rows)) return GB_ENOMEM;
    GB_CUDA_TRY(cudaMemcpyAsync(c->mx, hx, (size_t)cols * sizeof(float), cudaMemcpyHostToDevice, c->st));
    const int rc = gb_matvec(dtype, dW, rows, cols, c->mx, c->my, nullptr, c->st);
    if (rc) return rc;
    GB_CUDA_TRY(cudaMemcpyAsync(hy, c->my, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost, c->st));
    GB_CUDA_TRY(cudaStreamSynchronize(c->st));
    return GB_OK;
}

// The prepared matvec for device weights dW (re-planned if the shape changed),
// with the context's shared workspace grown to cover it.
static const MvPlan* plan_for(Ctx* c, int dtype, const void* dW, int rows, int cols, int* rc) {
    MvPlan& p = c->plans[dW];
    if (p.W != dW || p.dtype != dtype || p.rows != rows || p.cols != cols) {
        if ((*rc = mv_plan(&p, dtype, dW, rows, cols))) {
            c->plans.erase(dW);
            return nullptr;
        }
    }
    *rc = GB_OK;
    return &p;
}

// Grow the context's matvec workspace (zeroed in stream order) to `need`.
static int ensure_mv_ws(Ctx* c, size_t need) {
    if (need <= c->mv_ws_size) return GB_OK;
    if (c->mv_ws) {
        cudaStreamSynchronize(c->st);
        cudaFree(c->mv_ws);
        c->mv_ws = nullptr;
        c->mv_ws_size = 0;
    }
    if (cudaMalloc(&c->mv_ws, need) != cudaSuccess) {
        c->mv_ws = nullptr;
        return GB_ENOMEM;
    }
    if (cudaMemsetAsync(c->mv_ws, 0, need, c->st) != cudaSuccess) return GB_ECUDA;
    c->mv_ws_size = need;
    return GB_OK;
}

// FNV-1a over 64 words spread evenly through the buffer (and its last word).
// Byte cap of the vtable slots' cache of uploaded weights:
// GB_VTABLE_CACHE_MB in the environment, default 16384 (16 GiB).
static size_t vtable_cache_cap() {
    static const size_t v = [] {
        const char* e = getenv("GB_VTABLE_CACHE_MB");
        const long mb = e ? atol(e) : 16384;
        return (size_t)(mb > 0 ? mb : 16384) << 20;
    }();
    return v;
}

static uint64_t sample_signature(const void* p, size_t n) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    uint64_t h = 1469598103934665603ull ^ n;
    const size_t step = n / 64 > 8 ? n / 64 : 8;
    for (size_t off = 0; off + 8 <= n; off += step) {
        uint64_t w;
        memcpy(&w, b + off, 8);
        h = (h ^ w) * 1099511628211ull;
    }
    if (n >= 8) {
        uint64_t w;
        memcpy(&w, b + n - 8, 8);
        h = (h ^ w) * 1099511628211ull;
    }
    return h;
}

static int check_dtype_shape(int dtype, int rows, int cols) {
    if (rows <= 0 || cols <= 0) return GB_EINVAL;
    if (dtype != GB_DT_Q4_K && dtype != GB_DT_Q6_K && dtype != GB_DT_Q8_0 && dtype != GB_DT_Q5_K &&
        dtype != GB_DT_F16)
        return GB_EINVAL;
    if (cols % gb_block_width(dtype)) return GB_ESHAPE;
    return GB_OK;
}

}  // namespace gb

using namespace gb;

// ======================================================================= ABI
extern "C" void* cuda_upload_weight(const void* host_ptr, size_t size) {
    if (!host_ptr) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    return c ? upload_bytes(host_ptr, size, c->st) : nullptr;
}

extern "C" int cuda_matvec_q4k_f32_impl(const void* W_data, const float* x, float* y, int num_rows, int num_cols) {
    if (!W_data || !x || !y) return GB_EINVAL;
    int rc = check_dtype_shape(GB_DT_Q4_K, num_rows, num_cols);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return GB_ECUDA;
    return matvec_hostio(c, GB_DT_Q4_K, W_data, num_rows, num_cols, x, y);
}

// Host-buffer matvec for the vtable slots: W resident on the device (d_data)
// or, when it never was uploaded, uploaded once on first use and cached by its
// host pointer.  Error codes as the reference CPU kernels.
extern "C" __attribute__((visibility("hidden"))) int gb_vtable_matvec(int dtype, const void* host_data, const void* d_data, int resident,
                                size_t byte_size, int rows, int cols, const float* x, float* y) {
    if (!x || !y || (!host_data && !(resident && d_data))) return GB_EINVAL;
    // the reference kernels' order (quant_matvec_q4_k.c:150-158): columns not a
    // multiple of the block width, then the byte size when it is known.  An
    // empty matrix is no error there: no rows, nothing to do; no columns,
    // every row's sum is 0.  Negative shapes are rejected here (the reference
    // does not check them).
    if (dtype != GB_DT_Q4_K && dtype != GB_DT_Q6_K && dtype != GB_DT_Q8_0) return GB_EINVAL;
    if (rows < 0 || cols < 0) return GB_EINVAL;
    if (cols % gb_block_width(dtype)) return GB_ESHAPE;
    const size_t need = gb_matrix_bytes(dtype, rows, cols);
    if (byte_size != 0 && need > byte_size) return GB_ESIZE;
    if (rows == 0 || cols == 0) {
        if (rows > 0) memset(y, 0, (size_t)rows * sizeof(float));
        return GB_OK;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return GB_ECUDA;
    const void* dW = (resident && d_data) ? d_data : nullptr;
    if (!dW) {
        // A cached copy is reused only for the same size and sampled content:
        // a host buffer freed and reallocated at the same address must not
        // pick up (or over-read) the old device copy.  An edit in place that
        // misses the sampled bytes is not seen: such callers clear the cache
        // (gb_vtable_cache_clear).  The cache holds at most
        // vtable_cache_cap() bytes; the least recently used copies go first.
        const uint64_t sig = sample_signature(host_data, need);
        Ctx::CachedWeight& e = c->weight_cache[host_data];
        if (!e.d || e.bytes != need || e.sig != sig) {
            cudaStreamSynchronize(c->st);   // no launch still reads a copy freed below
            if (e.d) {
                cudaFree(e.d);
                c->weight_cache_bytes -= e.bytes;
                e = Ctx::CachedWeight{};
            }
            while (c->weight_cache_bytes + need > vtable_cache_cap() && c->weight_cache_bytes > 0) {
                auto lru = c->weight_cache.end();
                for (auto it = c->weight_cache.begin(); it != c->weight_cache.end(); ++it)
                    if (it->second.d && (lru == c->weight_cache.end() || it->second.last_use < lru->second.last_use))
                        lru = it;
                if (lru == c->weight_cache.end()) break;
                cudaFree(lru->second.d);
                c->weight_cache_bytes -= lru->second.bytes;
                c->weight_cache.erase(lru);
            }
            Ctx::CachedWeight& f = c->weight_cache[host_data];   // the erase above may have moved it
            void* d = upload_bytes(host_data, need, c->st);
            if (!d) {
                c->weight_cache.erase(host_data);
                return GB_ENOMEM;
            }
            f.d = d;
            f.bytes = need;
            f.sig = sig;
            c->weight_cache_bytes += need;
        }
        Ctx::CachedWeight& g = c->weight_cache[host_data];
        g.last_use = ++c->use_clock;
        dW = g.d;
    }
    return matvec_hostio(c, dtype, dW, rows, cols, x, y);
}

extern "C" int gb_vtable_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return GB_ECUDA;
    cudaStreamSynchronize(c->st);
    for (auto& kv : c->weight_cache)
        if (kv.second.d) cudaFree(kv.second.d);
    c->weight_cache.clear();
    c->weight_cache_bytes = 0;
    return GB_OK;
}

// Native host-buffer entry (same path as the vtable slots, device W).
extern "C" int gb_matvec_host(int dtype, const void* dW, int rows, int cols, const float* h_x, float* h_y) {
    if (!dW || !h_x || !h_y) return GB_EINVAL;
    int rc = check_dtype_shape(dtype, rows, cols);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return GB_ECUDA;
    return matvec_hostio(c, dtype, dW, rows, cols, h_x, h_y);
}

extern "C" int cuda_transformer_layer_gpu(
    const void* wq, int wq_rows, int wq_cols, int wq_dtype,
    const void* wk, int wk_rows, int wk_cols, int wk_dtype,
    const void* wv, int wv_rows, int wv_cols, int wv_dtype,
    const void* wo, int wo_rows, int wo_cols, int wo_dtype,
    const void* w_gate, int gate_rows, int gate_cols, int gate_dtype,
    const void* w_up, int up_rows, int up_cols, int up_dtype,
    const void* w_down, int down_rows, int down_cols, int down_dtype,
    const float* h_rms_att, const float* h_rms_ffn,
    float* h_hidden,
    float* h_k_cache, float* h_v_cache, int head_stride,
    int H, int n_heads, int n_kv_heads, int head_dim,
    int pos, int layer, int max_seq_len) {
    const void* W[GB_NMAT] = {wq, wk, wv, wo, w_gate, w_up, w_down};
    const int R[GB_NMAT] = {wq_rows, wk_rows, wv_rows, wo_rows, gate_rows, up_rows, down_rows};
    const int Cc[GB_NMAT] = {wq_cols, wk_cols, wv_cols, wo_cols, gate_cols, up_cols, down_cols};
    const int D[GB_NMAT] = {wq_dtype, wk_dtype, wv_dtype, wo_dtype, gate_dtype, up_dtype, down_dtype};
    if (!h_rms_att || !h_rms_ffn || !h_hidden || !h_k_cache || !h_v_cache) return GB_EINVAL;
    if (H <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0) return GB_EINVAL;
    if (pos < 0 || pos >= max_seq_len) return GB_EPOS;
    if (head_stride != max_seq_len * head_dim) return GB_EINVAL;
    const int KV = n_kv_heads * head_dim, F = gate_rows;
    const int want_rows[GB_NMAT] = {n_heads * head_dim, KV, KV, H, F, F, H};
    const int want_cols[GB_NMAT] = {H, H, H, n_heads * head_dim, H, H, F};
    for (int i = 0; i < GB_NMAT; i++) {
        if (!W[i]) return GB_EINVAL;
        int rc = check_dtype_shape(D[i], R[i], Cc[i]);
        if (rc) return rc;
        if (R[i] != want_rows[i] || Cc[i] != want_cols[i]) return GB_EINVAL;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return GB_ECUDA;
    if (!ensure_acts(c, H, KV, F) || !ensure_rope(c, max_seq_len, head_dim) ||
        !ensure_ws(c, n_heads, n_kv_heads, head_dim, max_seq_len))
        return GB_ENOMEM;
    LayerKV* L = layer_kv(c, layer, n_kv_heads, head_dim, max_seq_len);
    if (!L) return GB_ENOMEM;
    int rc;
    if (pos < L->valid) {   // a rewind (new conversation, restored session): the host cache is the truth
        if (pos > 0 && (rc = upload_kv(c, L, h_k_cache, h_v_cache, head_stride, 0, pos))) return rc;
        L->valid = pos;
    } else if (L->valid < pos) {   // positions computed elsewhere (CPU prefill, session load)
        if ((rc = upload_kv(c, L, h_k_cache, h_v_cache, head_stride, L->valid, pos))) return rc;
        L->valid = pos;
    }
    const float* ra = cached_norm(c, h_rms_att, H);
    const float* rf = cached_norm(c, h_rms_ffn, H);
    if (!ra || !rf) return GB_ENOMEM;
    GB_CUDA_TRY(cudaMemcpyAsync(c->hidden, h_hidden, (size_t)H * sizeof(float), cudaMemcpyHostToDevice, c->st));
    if ((rc = set_device_int(c->d_pos, pos, c->st))) return rc;
    LayerArgs a;
    for (int i = 0; i < GB_NMAT; i++)
        if (!(a.mv[i] = plan_for(c, D[i], W[i], R[i], Cc[i], &rc))) return rc;
    if ((rc = ensure_mv_ws(c, layer_ws_bytes(a.mv)))) return rc;
    a.mv_ws = c->mv_ws;
    a.ra = ra; a.rf = rf; a.kc = L->k; a.vc = L->v; a.rope = c->rope; a.d_pos = c->d_pos; a.attn_ws = c->ws;
    a.hidden = c->hidden; a.xn = c->xn; a.q = c->q; a.k = c->k; a.v = c->v; a.attn = c->attn;
    a.gate = c->gate; a.up = c->up;
    a.H = H; a.n_heads = n_heads; a.n_kv = n_kv_heads; a.hd = head_dim; a.ff = F; a.max_seq = max_seq_len;
    a.eps = 1e-6f;   // hard-coded by the reference (engine.c:359, 524)
    if ((rc = enqueue_layer(a, c->st))) return rc;
    GB_CUDA_TRY(cudaMemcpyAsync(h_hidden, c->hidden, (size_t)H * sizeof(float), cudaMemcpyDeviceToHost, c->st));
    // Keep the host cache coherent: copy the appended K/V row back.
    const size_t row = (size_t)head_dim * sizeof(float);
    const size_t dp = (size_t)max_seq_len * head_dim * sizeof(float), hp = (size_t)head_stride * sizeof(float);
    const size_t off = (size_t)pos * head_dim;
    GB_CUDA_TRY(cudaMemcpy2DAsync(h_k_cache + off, hp, L->k + off, dp, row, n_kv_heads, cudaMemcpyDeviceToHost, c->st));
    GB_CUDA_TRY(cudaMemcpy2DAsync(h_v_cache + off, hp, L->v + off, dp, row, n_kv_heads, cudaMemcpyDeviceToHost, c->st));
    L->valid = pos + 1;
    return GB_OK;
}

extern "C" void cuda_finish_layer(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (c && c->st) cudaStreamSynchronize(c->st);
}

extern "C" void cuda_sync_kv_cache(int layer, int n_kv_heads, int head_dim, int pos, int T, const float* h_k_cache,
                                   const float* h_v_cache, int stride0, int max_seq) {
    if (!h_k_cache || !h_v_cache || n_kv_heads <= 0 || head_dim <= 0 || pos < 0 || T <= 0 || max_seq <= 0) return;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = ctx();
    if (!c) return;
    LayerKV* L = layer_kv(c, layer, n_kv_heads, head_dim, max_seq);
    if (!L) return;
    // a sync below the mirrored positions is a rewind (a restored session or
    // prompt cache replaced the host K/V): upload the whole prefix again
    const bool rewind = pos < L->valid;
    const int p0 = rewind ? 0 : L->valid;
    const int p1 = pos + T < max_seq ? pos + T : max_seq;
    if (upload_kv(c, L, h_k_cache, h_v_cache, stride0, p0, p1) == GB_OK && (rewind || p1 > L->valid)) L->valid = p1;
}

// NVML read through dlopen (no link-time dependency); 0 when unavailable.
extern "C" int cuda_get_temperature(void) {
    typedef int (*init_t)(void);
    typedef int (*handle_t)(unsigned, void**);
    typedef int (*temp_t)(void*, int, unsigned*);
    static void* lib = nullptr;
    static init_t init = nullptr;
    static handle_t handle = nullptr;
    static temp_t temp = nullptr;
    static int state = 0;   // 0 untried, 1 ok, -1 unavailable
    std::lock_guard<std::mutex> lk(g_mu);
    if (state == 0) {
        lib = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
        if (lib) {
            init = (init_t)dlsym(lib, "nvmlInit_v2");
            handle = (handle_t)dlsym(lib, "nvmlDeviceGetHandleByIndex_v2");
            temp = (temp_t)dlsym(lib, "nvmlDeviceGetTemperature");
        }
        state = (init && handle && temp && init() == 0) ? 1 : -1;
    }
    if (state != 1) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    void* h = nullptr;
    unsigned t = 0;
    if (handle((unsigned)dev, &h) != 0 || temp(h, 0 /* NVML_TEMPERATURE_GPU */, &t) != 0) return 0;
    return (int)t;
}
