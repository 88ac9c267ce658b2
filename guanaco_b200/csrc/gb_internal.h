// gb_internal.h -- host-side declarations shared between the library's
// translation units (not part of the public ABI).
#pragma once

#include "../../include/guanaco_b200.h"
#include <cuda_runtime.h>

namespace gb {

// SM count of the current device (queried once per device).
int sm_count();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize, bytes) once per
// (kernel, device); thread-safe.
cudaError_t set_smem_once(const void* func, int bytes);

// Attention split geometry shared by the launcher and the workspace sizing:
// the grid has n_kv * grid_splits CTAs; each covers P consecutive positions,
// P chosen in-kernel from pos so that the active splits fit the grid.
int attn_grid_splits(int n_kv, int max_seq);
// gb_attention_decode, and when xq_out != nullptr also the output quantised
// for a matvec that reads it pre-quantised (MV_X_PREQ): the CTA that finishes
// a KV head quantises each 32-column group of that head group's output
// (mt_quantise32 layout, n_heads * head_dim columns, a multiple of 256).
// pdl: the decode step's launch after its q/k/v matvec (which writes neither
// the caches nor the position) may start early and stream the cached K / V.
int attention_decode_xq(const float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                        const float* rope_cs, const int* d_pos, int n_heads, int n_kv, int head_dim, int max_seq,
                        float* out, void* ws, uint8_t* xq_out, cudaStream_t st, bool pdl = false);

// A prepared matvec: kernel choice, launch geometry and, for the TMA path,
// the encoded tensor map of W.  Built once per weight matrix on the host
// (the map holds W's address, so a plan is tied to one device buffer).
struct MvPlan {
    alignas(64) unsigned char tmap[128];   // CUtensorMap for the TMA kernels
    const void* W = nullptr;
    int dtype = 0, rows = 0, cols = 0, nb = 0;
    int kind = 0;                          // MV_RING or MV_TMA
    int nch = 0, T = 0, ncta = 0, S = 0, ngroups = 0;
    size_t smem = 0;
};
enum { MV_RING = 0, MV_TMA = 1 };
int mv_plan(MvPlan* p, int dtype, const void* W, int rows, int cols);
// Device workspace the plan's launches need (stream-K partials + per-group
// tickets).  Zero it once; every launch leaves the tickets at zero again.
// Launches that share a workspace must not overlap in time.
size_t mv_ws_bytes(const MvPlan& p);
// ws may be null: the TMA path then splits the rows by whole groups (no
// cross-CTA partials, less even for short matrices).  pdl: launch with
// programmatic stream serialization, so the kernel's weight prefetch overlaps
// the tail of the previous kernel on the stream.
// Optional transform of x inside the matvec (TMA path only): RMSNorm
// x * r * w (r = 1 / sqrt(mean(x^2) + eps), the reference's rounding), or
// silu(x) * x2 (the SwiGLU product).
// MV_X_PREQ: x arrives already quantised (xq, the layout the x quantiser
// writes in shared memory, mt_xq_bytes(K, true) bytes).
enum { MV_X_NONE = 0, MV_X_RMSNORM = 1, MV_X_SILU_MUL = 2, MV_X_PREQ = 3 };
struct MvXform {
    int mode = MV_X_NONE;
    const float* w = nullptr;    // RMSNorm weight
    const float* x2 = nullptr;   // the up projection for MV_X_SILU_MUL
    float eps = 0.f;
    const uint8_t* xq = nullptr;   // MV_X_PREQ input
    // gate / up launch (two matrices of equal rows, one item per 32-row
    // group): silu(y0) * y1 is also quantised into swq_out (mt_xq_bytes(rows,
    // true) bytes, zero-initialised) for the ffn_down matvec; swq_tk holds one
    // ticket per group (zero between launches)
    uint8_t* swq_out = nullptr;
    unsigned* swq_tk = nullptr;
    int swq_K = 0;                 // columns of swq_out (the ffn_down K, >= rows, a multiple of 256)
};
// Tensor-parallel exchange attached to a TMA matvec launch (world > 1).
// Every rank owns a receive buffer whose first part is slots[2][world][H]
// of {value bits, epoch} pairs (8-byte stores, so a value is valid once its
// epoch tag matches: no flag, no fence); the peers write it over NVLink
// through CUDA IPC mappings.  Exchange c of a step has epoch
// step * calls + c + 1 and uses slot parity epoch & 1.
//   push_call >= 0: the launch's y rows (one matrix, no residual) go to slot
//                   [rank] of every rank's buffer instead of y.
//   in_call >= 0:   x (RMSNorm input) = x + sum over ranks, in rank order,
//                   of this rank's slots of exchange in_call (bounded waits
//                   for the tags); h_out receives the new hidden state.
//                   Slice form (ready != null): CTA c sums only its slice of
//                   x, writes it to h_out and releases ready[c] = epoch;
//                   every CTA then waits (bounded) for all ready flags and
//                   reads the whole new hidden state from h_out, so the slots
//                   are read once per rank.  Direct form (ready == null):
//                   every CTA sums all slots itself and writes its slice of
//                   h_out -- no grid-wide wait, world x H slot reads per CTA.
struct MvTp {
    void* const* peers = nullptr;               // device array of the ranks' receive buffers
    const unsigned long long* step = nullptr;   // device step counter
    unsigned* err = nullptr;                    // device error word (GB_ETIMEOUT)
    unsigned* ready = nullptr;                  // slice form: this rank's per-CTA flags (GB_MAX_SMS, zeroed once)
    int rank = 0, world = 1, calls = 0, H = 0;
    int push_call = -1, in_call = -1;
    float* h_out = nullptr;
};
int mv_launch(const MvPlan& p, const float* x, float* y, const float* residual, void* ws, cudaStream_t st,
              bool pdl, const MvXform* xf = nullptr, const MvTp* tp = nullptr);
// Several matrices that share x as one launch (TMA plans of one format, one
// column count and ring depth; at most 3): ys[i] = W_i x (+ res[i]).
bool mv_groupable(const MvPlan* const* ps, int n);
size_t mv_ws_bytes_group(const MvPlan* const* ps, int n);
int mv_launch_group(const MvPlan* const* ps, int n, const float* x, float* const* ys, const float* const* res,
                    void* ws, cudaStream_t st, bool pdl, const MvXform* xf = nullptr, const MvTp* tp = nullptr);
// Tensor map of a Q4_K / Q6_K weight view (gb_matvec.cu).
bool mt_encode_view(void* map128, int dtype, const void* W, int rows, int nb, int boxz);
bool mt_encode_rows(void* map128, const void* W, int rows, int nb, int box_u64);
// Tensor map of a row-major fp32 matrix X[T][K] with boxes {box_k columns,
// box_t rows, 1}; rows past T read as zeros.  X and the row pitch 16-byte aligned.
bool gemm_encode_x(void* map128, const float* X, int T, int K, int box_k, int box_t);
bool gemm_encode_x16(void* map128, const void* X16, int Tp, int K, int box_t);

// A GEMM's activations split for fp16 operands (gemm_split_x): X * 2^e_t =
// hi + lo, rows scaled so that max |x| < 2^15, hi and lo each laid out
// [K / 8][tp][8] halves (column group, token, column; tp = T rounded up to a
// multiple of 256, rows past T zero), and inv[t] = 2^-e_t.
struct GemmX16 {
    const void* hi;
    const void* lo;
    const float* inv;
    int tp;
};
inline int gemm_split_rows(int T) { return (T + 255) / 256 * 256; }
// Prefill GEMM on the tensor cores (gb_gemm.cu): Y[t][n] = sum_k X[t][k]
// W[n][k] (+ R[t][n]) for T tokens, W fp32 (dtype GB_DT_F32) or GGUF blocks;
// fp32-equivalent (3xF16, or 3xTF32 with GB_GEMM_KIND=tf32).  R may alias Y.
// A wait that gives up records GB_ETIMEOUT in *err (null: the module-wide
// word of gb_gemm_error).  Rows of Y and R are ldy floats apart (0: N).
// x16: X already split (shared by GEMMs of one X); null splits X into
// stream-ordered scratch first.
int gemm_launch(int dtype, const void* W, const float* X, float* Y, const float* R, int N, int K, int T,
                cudaStream_t st, unsigned* err = nullptr, int ldy = 0, const GemmX16* x16 = nullptr);
// Y[t][f] = silu(X Wg^T)[t][f] * (X Wu^T)[t][f] (k_silu_mul's rounding) for
// f < F, in one GEMM launch: gate and up (same dtype, F rows each) share the
// activation tiles, and the two products never reach HBM.
int gemm_swiglu_launch(int dtype, const void* Wg, const void* Wu, const float* X, float* Y, int F, int K, int T,
                       cudaStream_t st, unsigned* err = nullptr, int ldy = 0, const GemmX16* x16 = nullptr);
// True unless GB_GEMM_KIND=tf32: the GEMMs take split activations.
bool gemm_f16_operands();
// Split X [T][K] (rows K floats apart, K a multiple of 32) for fp16 operands
// into hi / lo (gemm_split_rows(T) x K halves each) and inv (T floats).
int gemm_split_x(const float* X, int T, int K, void* hi, void* lo, float* inv, cudaStream_t st);
// The split of RMSNorm(X) rows (weight w, may be null) without writing them:
// rmsnorm_rows followed by gemm_split_x in one pass.
int gemm_rmsnorm_split_x(const float* X, const float* w, int T, int K, float eps, void* hi, void* lo, float* inv,
                         cudaStream_t st);

// Tensor-parallel context of a layer (world > 1): the wo and ffn_down
// matvecs write this rank's partial to `part`, then an all-reduce over peer
// memory adds every rank's partial to the hidden state.
struct TpCtx {
    int rank = 0, world = 1;
    void* const* d_peers = nullptr;          // device array: every rank's exchange buffer
    const unsigned long long* d_step = nullptr;
    int calls = 0;                            // exchanges per step
    unsigned* err = nullptr;
    unsigned* ready = nullptr;                // per-CTA slice flags of the in-matvec exchanges
    float* part = nullptr;                    // [H] local partial
    float* h[2] = {nullptr, nullptr};         // hidden state: exchange c reads h[c & 1], writes h[(c + 1) & 1]
    // an exchange attached to a matvec (push_call / in_call filled in by the caller)
    MvTp mv() const {
        MvTp t;
        t.peers = d_peers;
        t.step = d_step;
        t.err = err;
        t.ready = ready;
        t.rank = rank;
        t.world = world;
        t.calls = calls;
        return t;
    }
};
// Exchange `call` as its own launch: push part to every rank, then
// h_out = h_in + sum of the ranks' partials (rank order).
int tp_allreduce(const TpCtx& tp, const float* h_in, float* h_out, int H, int call, cudaStream_t st);

// Everything one decode layer needs; all pointers are device pointers.
struct LayerArgs {
    const TpCtx* tp = nullptr;   // null: one GPU
    int layer = 0;
    const MvPlan* mv[GB_NMAT];
    void* mv_ws;
    const float* ra;          // pre-attention RMSNorm weight
    const float* rf;          // pre-MLP RMSNorm weight
    float* kc;                // this layer's K cache [n_kv][max_seq][hd]
    float* vc;                // this layer's V cache
    const float* rope;        // RoPE table [max_seq][hd]
    const int* d_pos;
    void* attn_ws;
    float *hidden, *xn, *q, *k, *v, *attn, *gate, *up;
    int H, n_heads, n_kv, hd, ff, max_seq;
    float eps;
    bool tp_fused = false;    // tensor parallel: exchanges inside the matvecs (tp_fusable for every layer)
    // SwiGLU product quantised by the gate / up launch for ffn_down
    // (5 K / 2 bytes for K = ffn_down's columns, zeroed once) and its pair
    // tickets (K / 32, zero); null: ffn_down quantises it itself
    uint8_t* swq = nullptr;
    unsigned* swq_tk = nullptr;
    uint8_t* aq = nullptr;    // attention output quantised for wo (nullptr: wo quantises it)
};
int enqueue_layer(const LayerArgs& a, cudaStream_t st);
bool tp_fusable(const MvPlan* const* mv, int H);
// Matvec workspace one layer's launches need (grouped launches included).
size_t layer_ws_bytes(const MvPlan* const* mv);
// Embedding rows of d_token[0 .. rows) into out[rows][H].
int embed(const void* emb, int dtype, const int* d_token, int vocab, int H, float* out, unsigned* err,
          cudaStream_t st, unsigned long long* step = nullptr, int rows = 1);
// out[r] = RMSNorm(x[r]) * w for rows r < rows of n elements.
int rmsnorm_rows(const float* x, const float* w, float* out, int n, int rows, float eps, cudaStream_t st);
int set_device_int(int* p, int v, cudaStream_t st);

// Everything one prefill layer needs (gb_prefill.cu): T prompt tokens at
// positions pos0 .. pos0 + T - 1, activations row-major [T][width].
struct PrefillArgs {
    const void* w[GB_NMAT];   // whole matrices (one GPU)
    int dt[GB_NMAT];
    const float *ra, *rf;     // RMSNorm weights
    float *kc, *vc;           // this layer's caches [n_kv][max_seq][hd]
    const float* rope;        // RoPE table [max_seq][hd]
    float *hidden, *xn, *q, *k, *v, *attn, *gate, *up;
    void *xh, *xl;            // [T][K] fp16 halves of the current GEMM input (fp16 operands)
    float* xinv;              // [T] its token scales' inverses
    cudaStream_t side;        // wk / wv run here beside wq (null: all on the layer's stream)
    cudaEvent_t fork, join;
    unsigned* err;            // the model's error word
    int T, pos0, H, n_heads, n_kv, hd, ff, max_seq;
    int fk;                   // ffn_down's columns (ff, or ff rounded up with zero padding): gate / up row width
    float eps;
};
int enqueue_prefill_layer(const PrefillArgs& a, cudaStream_t st);
// Causal attention of T query rows (positions pos0 ..) over the cache.
// Timeouts of its bounded waits go to *err (null: the module word read by
// gb_prefill_attention_error).
int prefill_attention(const float* q, const float* kc, const float* vc, float* out, int T, int pos0, int n_heads,
                      int n_kv, int head_dim, int max_seq, cudaStream_t st, unsigned* err);
// Synthetic blocks of a slice of a larger matrix: local block r * sn + j
// (r < rows, j < sn) is global block (row0 + r) * nbg + c0 + j of stream
// stream_id, written at out block r * ldo + j (ldo >= sn; blocks j >= sn of a
// row are left untouched).
int synth_blocks_shard(int dtype, void* out, size_t rows, size_t sn, size_t ldo, uint64_t row0, uint64_t nbg,
                       uint64_t c0, uint64_t seed, uint64_t stream_id, cudaStream_t st);

}  // namespace gb
