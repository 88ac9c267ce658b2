#!/usr/bin/env python3
"""Decode throughput of the UNCHANGED reference engine with this library as its
CUDA backend (test infrastructure, like the rest of oracle/: never part of
the product, never imported by the product or by bench.py's timed arms).

    python oracle/engine_dropin_bench.py [--warmup W] [--steps K] [--layers L]

Loads oracle/_ref/libref_dropin.so -- src/engine/engine.c and the reference's
CPU kernels, backend factory and KV cache compiled with -DUSE_CUDA=1 and
linked against guanaco_b200/lib/libguanaco_b200.so -- builds the
Llama-3.1-8B-shape synthetic model (seeded, Q4_K with Q6_K for attn_v,
ffn_down and the output head; the seeds and streams of gb_model_synthesize),
fills K / V to 4096 positions, moves the layers to the device as the engine's
loader does (cuda_upload_weight, device_residency = 1) and times forward()
for single tokens: 32 x cuda_transformer_layer_gpu with the host hidden
state in and out per layer, then the CPU final RMSNorm and the output head
through the vtable slot of backend_create(AUTO).  Prints one JSON line.
Needs one GPU.
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

SEED = 1234
CTX = 4096


def engine_dropin_tokens_per_s(warmup: int = 3, steps: int = 32, n_layers: int = 32) -> dict:
    import numpy as np
    import torch

    import guanaco_b200 as gb
    from oracle import oracle as O
    from tests.synth_model import fill_kv, gpu_blocks, synth_model

    if not O.dropin_available():
        return {"engine_dropin": {"unavailable": "oracle/_ref/libref_dropin.so not built (needs the reference tree)"}}
    torch.cuda.set_device(0)
    gb.lib()
    threads = os.cpu_count() or 1
    m = synth_model(O, 4096, 32, 8, n_layers, 14336, 128256, CTX + warmup + steps + 8, SEED,
                    gen=gpu_blocks(gb, torch))
    eng = O.RefModel(m, lib=O.dropin())
    try:
        O.dropin().ref_set_threads(threads)
        fill_kv(O, eng, m, CTX, SEED)
        eng.to_gpu(threads)
        token, pos = 1, CTX
        for _ in range(warmup):
            token = int(np.argmax(eng.forward(token, pos)))
            pos += 1
        t0 = time.perf_counter()
        toks = []
        for _ in range(steps):
            token = int(np.argmax(eng.forward(token, pos)))
            toks.append(token)
            pos += 1
        dt = time.perf_counter() - t0
    finally:
        eng.close()
    return {"engine_dropin": {
        "tokens_per_s": round(steps / dt, 2), "ms_per_token": round(dt / steps * 1e3, 3),
        "layers": n_layers, "positions": [CTX + warmup, CTX + warmup + steps - 1], "host_threads": threads,
        "path": "reference engine forward() (-DUSE_CUDA=1) -> cuda_transformer_layer_gpu x layers (host hidden "
                "in/out) -> CPU RMSNorm -> vtable matvec_q6k_f32 output head -> host argmax",
        "timing": "host wall clock per forward() call"}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--layers", type=int, default=32)
    a = ap.parse_args()
    print(json.dumps(engine_dropin_tokens_per_s(a.warmup, a.steps, a.layers)), flush=True)


if __name__ == "__main__":
    main()
