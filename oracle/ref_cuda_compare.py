#!/usr/bin/env python3
"""GPU comparison against the reference's own CUDA path (test
infrastructure, like the rest of oracle/: never part of the product).

    python oracle/ref_cuda_compare.py [--warmup W] [--steps K]

Loads oracle/_ref/libref_cuda.so (the reference's cuda_layer_kernels.cu and
matvec_q4k_cuda.cu compiled unchanged for sm_100a by oracle/Makefile) beside
guanaco_b200's library and prints one JSON line.  Needs one GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# run as a script, this file's directory would shadow the oracle package
sys.path = [ROOT] + [p for p in sys.path if os.path.abspath(p or ".") != os.path.join(ROOT, "oracle")]

LLAMA8B = dict(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=32, ff_dim=14336, vocab_size=128256)
SEED = 1234


def ref_cuda_compare(warmup: int = 4, steps: int = 16) -> dict:
    """The reference's own CUDA path (src/kernels/cuda/cuda_layer_kernels.cu,
    matvec_q4k_cuda.cu, compiled unchanged for sm_100a into
    oracle/_ref/libref_cuda.so) beside this library, both through the
    engine-facing ABI: cuda_transformer_layer_gpu for the 32 Llama-8B layers of
    one token (host hidden in / out, then cuda_finish_layer, as engine.c calls
    it) and cuda_matvec_q4k_f32_impl (host x / y) on config 0.  The reference
    keeps at most 2048 positions in VRAM (cuda_layer_kernels.cu:407-410), so
    the tokens run at positions just below 2048; its K / V history is uploaded
    with its cuda_sync_kv_cache first.  Wall-clock on the host for both arms,
    synthetic seeded weights and K / V."""
    import ctypes as C

    import numpy as np
    import torch

    import guanaco_b200 as gb
    from oracle import oracle as O

    path = os.path.join(ROOT, "oracle", "_ref", "libref_cuda.so")
    if not os.path.exists(path):
        return {"ref_cuda": {"unavailable": "oracle/_ref/libref_cuda.so not built (needs the reference tree)"}}
    torch.cuda.set_device(0)
    ours = gb.lib()
    ref = C.CDLL(path, mode=os.RTLD_LOCAL | getattr(os, "RTLD_DEEPBIND", 0))
    vp, i = C.c_void_p, C.c_int
    for L in (ref,):
        L.cuda_transformer_layer_gpu.restype = i
        L.cuda_transformer_layer_gpu.argtypes = [vp, i, i, i] * 7 + [vp] * 5 + [i] * 8
        L.cuda_finish_layer.restype = None
        L.cuda_finish_layer.argtypes = []
        L.cuda_sync_kv_cache.restype = None
        L.cuda_sync_kv_cache.argtypes = [i, i, i, i, i, vp, vp, i, i]
        L.cuda_matvec_q4k_f32_impl.restype = i
        L.cuda_matvec_q4k_f32_impl.argtypes = [vp, vp, vp, i, i]
    c = LLAMA8B
    H, nh, nkv, ff, NL = c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["ff_dim"], c["n_layers"]
    hd, ms = H // nh, 2048
    kvd = nkv * hd
    shapes = [(H, H, 4), (kvd, H, 4), (kvd, H, 5), (H, H, 4), (ff, H, 4), (ff, H, 4), (H, ff, 5)]
    layers = []
    for l in range(NL):
        ws = []
        for j, (r, cc, dt) in enumerate(shapes):
            nbytes = gb.matrix_bytes(dt, r, cc)
            t = torch.empty(nbytes + 16, dtype=torch.uint8, device="cuda")
            gb.synth_blocks(dt, t, nbytes // gb.BLOCK_BYTES[dt], SEED, 2000 + 10 * l + j)
            ws.append(t)
        layers.append(ws)
    torch.cuda.synchronize()
    ra = (1.0 + 0.01 * O.synth_normal(H, SEED, 40)).astype(np.float32)
    rf = (1.0 + 0.01 * O.synth_normal(H, SEED, 41)).astype(np.float32)
    W, K = max(2, warmup), max(4, steps)
    pos0 = ms - W - K - 1
    kv_host = O.synth_normal(nkv * ms * hd, SEED, 42).reshape(nkv, ms, hd)
    kv_host[:, pos0:] = 0.0

    def run(L, sync_first):
        kcs = [np.ascontiguousarray(kv_host.copy()).ravel() for _ in range(NL)]
        vcs = [np.ascontiguousarray(kv_host.copy()).ravel() for _ in range(NL)]
        if sync_first:
            for l in range(NL):
                L.cuda_sync_kv_cache(l, nkv, hd, 0, pos0, kcs[l].ctypes.data, vcs[l].ctypes.data, ms * hd, ms)
        h = O.synth_normal(H, SEED, 43)
        outs, t = [], None
        for step in range(W + K):
            if step == W:
                L.cuda_finish_layer()
                t = time.perf_counter()
            pos = pos0 + step
            for l in range(NL):
                a = []
                for w, (r, cc, dt) in zip(layers[l], shapes):
                    a += [w.data_ptr(), r, cc, dt]
                rc = L.cuda_transformer_layer_gpu(*a, ra.ctypes.data, rf.ctypes.data, h.ctypes.data,
                                                  kcs[l].ctypes.data, vcs[l].ctypes.data, ms * hd, H, nh, nkv,
                                                  hd, pos, l, ms)
                if rc != 0:
                    raise RuntimeError(f"cuda_transformer_layer_gpu returned {rc}")
            L.cuda_finish_layer()
            outs.append(h.copy())
        dt_s = time.perf_counter() - t
        return K / dt_s, outs

    tps_ref, h_ref = run(ref, True)
    tps_ours, h_ours = run(ours, False)
    rel = float(np.linalg.norm(h_ours[0].astype(np.float64) - h_ref[0]) /
                max(np.linalg.norm(h_ref[0].astype(np.float64)), 1e-30))

    # config 0 through the host-buffer matvec entry both libraries export
    rows = cols = 4096
    Wq = layers[0][0]
    x = O.synth_normal(cols, SEED, 44)
    res = {}
    for name, L in (("reference", ref), ("ours", ours)):
        y = np.zeros(rows, np.float32)
        for _ in range(3):
            L.cuda_matvec_q4k_f32_impl(Wq.data_ptr(), x.ctypes.data, y.ctypes.data, rows, cols)
        n = 50
        t = time.perf_counter()
        for _ in range(n):
            rc = L.cuda_matvec_q4k_f32_impl(Wq.data_ptr(), x.ctypes.data, y.ctypes.data, rows, cols)
        res[name] = round((time.perf_counter() - t) / n * 1e6, 2)
        if rc != 0:
            raise RuntimeError(f"cuda_matvec_q4k_f32_impl returned {rc}")
    return {"ref_cuda": {
        "layer_abi_tokens_per_s": {"reference": round(tps_ref, 3), "ours": round(tps_ours, 3)},
        "positions": [pos0 + W, pos0 + W + K - 1], "layers": NL, "output_head": "not included (engine.c runs it)",
        "hidden_rel_l2_first_token": rel,
        "matvec_q4k_impl_us_4096x4096": res,
        "timing": "host wall clock; reference and this library through the same extern C entry points"}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--steps", type=int, default=16)
    a = ap.parse_args()
    # positions stay below the reference's 2048-slot VRAM cap
    if a.warmup + a.steps > 64:
        ap.error("--warmup + --steps must stay <= 64")
    print(json.dumps(ref_cuda_compare(a.warmup, a.steps)), flush=True)


if __name__ == "__main__":
    main()
