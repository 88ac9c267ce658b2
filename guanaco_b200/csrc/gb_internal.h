// gb_internal.h -- host-side declarations shared between the library's
// translation units (not part of the public ABI).
#pragma once

#include "../../include/guanaco_b200.h"
#include <cuda_runtime.h>

namespace gb {

// Attention split geometry shared by the launcher and the workspace sizing:
// the grid has n_kv * grid_splits CTAs; each covers P consecutive positions,
// P chosen in-kernel from pos so that the active splits fit the grid.
int attn_grid_splits(int n_kv, int max_seq);

// Everything one decode layer needs; all pointers are device pointers.
struct LayerArgs {
    const void* w[GB_NMAT];
    int dt[GB_NMAT];
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
};
int enqueue_layer(const LayerArgs& a, cudaStream_t st);
int embed(const void* emb, int dtype, const int* d_token, int vocab, int H, float* out, unsigned* err,
          cudaStream_t st);
int set_device_int(int* p, int v, cudaStream_t st);

}  // namespace gb
