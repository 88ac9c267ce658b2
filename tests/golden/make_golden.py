"""Generate the golden fixtures under tests/golden/ (run in the build
container, where the reference tree and oracle/_ref/libref.so exist).

golden.npz  -- known-answer tests restated from the reference's
               tests/test_quant.c and seeded vectors evaluated by the
               reference's own C kernels (oracle/_ref/libref.so, compiled
               unchanged from the reference sources by oracle/Makefile).
abi_layout.json -- sizeof / offsetof of the reference's Tensor,
               BackendConfig, KernelVTable and struct Backend, compiled from
               the reference headers.

Usage: python tests/golden/make_golden.py [--ref <reference checkout>]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

SEED = 1234
FP16_ONE, FP16_TWO = 0x3C00, 0x4000


def kat_blocks():
    """The blocks of tests/test_quant.c (26-242)."""
    k = {}
    # test_q8_0_matvec (26-68): scale 1.0 with quants 1..32, scale 2.0 with -1..-32
    b = np.zeros(2 * O.Q80_BYTES, dtype=np.uint8)
    b[0:2] = np.frombuffer(np.uint16(FP16_ONE).tobytes(), np.uint8)
    b[2:34] = np.arange(1, 33, dtype=np.int8).view(np.uint8)
    b[34:36] = np.frombuffer(np.uint16(FP16_TWO).tobytes(), np.uint8)
    b[36:68] = (-np.arange(1, 33, dtype=np.int16)).astype(np.int8).view(np.uint8)
    k["kat_q8_0_blocks"] = b
    k["kat_q8_0_x"] = np.ones(64, dtype=np.float32)
    # test_q4_k_matvec (94-139): d = 1, dmin = 0, scales bytes all 1, qs = 0x12
    b = np.zeros(O.Q4K_BYTES, dtype=np.uint8)
    b[0:2] = np.frombuffer(np.uint16(FP16_ONE).tobytes(), np.uint8)
    b[4:16] = 1
    b[16:144] = 0x12
    k["kat_q4k_uniform_blocks"] = b
    k["kat_q4k_uniform_x"] = np.ones(256, dtype=np.float32)
    # test_q4_k_scales_and_nibbles_mapping (159-218): cross-byte 6-bit packing
    b = np.zeros(O.Q4K_BYTES, dtype=np.uint8)
    b[0:2] = np.frombuffer(np.uint16(FP16_ONE).tobytes(), np.uint8)
    b[2:4] = np.frombuffer(np.uint16(FP16_ONE).tobytes(), np.uint8)
    b[4:16] = [0xC1, 0x42, 0x85, 0x0F, 0xF0, 0x3C, 0x83, 0x55, 0x12, 0x34, 0x56, 0x78]
    b[16 + 0] = (2 << 4) | 1
    b[16 + 32] = (4 << 4) | 3
    b[16 + 64] = (6 << 4) | 5
    b[16 + 96] = (8 << 4) | 7
    x = np.zeros(256, dtype=np.float32)
    x[[0, 32, 64, 96, 128, 160, 192, 224]] = 1.0
    k["kat_q4k_mapping_blocks"] = b
    k["kat_q4k_mapping_x"] = x
    return k


def kat_mapping_expected(sc):
    """The test's independent restatement (test_quant.c:141-157, 204-210)."""
    def su6(g):
        return sc[g] & 0x3F if g < 4 else (sc[g + 4] & 0x0F) | (((sc[g - 4] >> 6) & 3) << 4)

    def mu6(g):
        return sc[g + 4] & 0x3F if g < 4 else ((sc[g + 4] >> 4) & 0x0F) | (((sc[g] >> 6) & 3) << 4)
    return float(sum(su6(g) * (g + 1) - mu6(g) for g in range(8)))


SHAPES = {O.DT_Q4_K: [(1, 256), (7, 512), (33, 1024), (64, 2048)],
          O.DT_Q6_K: [(1, 256), (7, 512), (33, 1024), (64, 2048), (5, 5632)],
          O.DT_Q8_0: [(1, 32), (7, 96), (33, 1024), (64, 2048)]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GUANACO_REF", os.path.join(ROOT, "..", "reference")),
                    help="reference checkout (default: $GUANACO_REF, else ../reference beside the repository)")
    a = ap.parse_args()
    O.build()
    if not O.ref_available():
        sys.exit("oracle/_ref/libref.so missing: the reference tree is needed to make fixtures")
    out = kat_blocks()
    R = O.ref()
    R.ref_set_threads(1)
    rc, y = O.ref_matvec(O.DT_Q8_0, out["kat_q8_0_blocks"], 1, 64, out["kat_q8_0_x"])
    assert rc == 0 and y[0] == -528.0, y
    out["kat_q8_0_expected"] = np.float32([-528.0])
    rc, y = O.ref_matvec(O.DT_Q4_K, out["kat_q4k_uniform_blocks"], 1, 256, out["kat_q4k_uniform_x"])
    assert rc == 0 and y[0] == 384.0, y
    out["kat_q4k_uniform_expected"] = np.float32([384.0])
    exp = kat_mapping_expected(out["kat_q4k_mapping_blocks"][4:16].astype(np.int64))
    rc, y = O.ref_matvec(O.DT_Q4_K, out["kat_q4k_mapping_blocks"], 1, 256, out["kat_q4k_mapping_x"])
    assert rc == 0 and abs(y[0] - exp) <= 1e-4, (y, exp)
    out["kat_q4k_mapping_expected"] = np.float32([exp])

    # Seeded vectors through the reference's own kernels.
    for dt, shapes in SHAPES.items():
        for si, (rows, cols) in enumerate(shapes):
            W = O.synth_blocks(dt, rows, cols, SEED, 100 + si)
            x = O.synth_normal(cols, SEED, 200 + si)
            rc, y = O.ref_matvec(dt, W, rows, cols, x)
            assert rc == 0
            tag = f"mv_{dt}_{rows}x{cols}"
            out[tag + "_W"] = W
            out[tag + "_x"] = x
            out[tag + "_y"] = y
    for dt in (O.DT_Q4_K, O.DT_Q8_0):
        B = O.synth_blocks(dt, 2, 512, SEED, 300)
        out[f"dq_{dt}_blocks"] = B
        out[f"dq_{dt}_out"] = O.ref_dequant(dt, B)
    # Attention step (RoPE + append + GQA attention) on the reference kernels.
    for name, (nh, nkv, hd, ms, pos) in {"attn_a": (8, 2, 128, 80, 67), "attn_b": (8, 1, 64, 40, 0),
                                         "attn_c": (16, 2, 64, 130, 129)}.items():
        q = O.synth_normal(nh * hd, SEED, 400)
        k = O.synth_normal(nkv * hd, SEED, 401)
        v = O.synth_normal(nkv * hd, SEED, 402)
        kc = O.synth_normal(nkv * ms * hd, SEED, 403)
        vc = O.synth_normal(nkv * ms * hd, SEED, 404)
        o, kc2, vc2 = O.ref_attention_step(q, k, v, kc, vc, nh, nkv, hd, ms, pos)
        out[name + "_dims"] = np.int32([nh, nkv, hd, ms, pos])
        out[name + "_out"] = o
        out[name + "_krow"] = kc2.reshape(nkv, ms, hd)[:, pos, :].copy()
        out[name + "_vrow"] = vc2.reshape(nkv, ms, hd)[:, pos, :].copy()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)

    # ABI layout of the reference structs.
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "backend_internal.h"
#define F(T, f) printf("\"%s.%s\": %zu,\n", #T, #f, offsetof(T, f))
int main(void) {
  printf("{\n");
  printf("\"sizeof.Tensor\": %zu,\n", sizeof(Tensor));
  F(Tensor, data); F(Tensor, shape); F(Tensor, stride); F(Tensor, ndim); F(Tensor, dtype);
  F(Tensor, ggml_type); F(Tensor, byte_size); F(Tensor, device_residency); F(Tensor, d_data);
  printf("\"sizeof.BackendConfig\": %zu,\n", sizeof(BackendConfig));
  F(BackendConfig, kind); F(BackendConfig, threads); F(BackendConfig, device_id); F(BackendConfig, n_gpu_layers);
  printf("\"sizeof.KernelVTable\": %zu,\n", sizeof(KernelVTable));
  F(KernelVTable, gemm_f32); F(KernelVTable, elemwise_mul); F(KernelVTable, matvec_q4k_f32);
  F(KernelVTable, matvec_q6k_f32); F(KernelVTable, matvec_q8_0_f32);
  printf("\"sizeof.Backend\": %zu,\n", sizeof(struct Backend));
  printf("\"Backend.cfg\": %zu,\n", offsetof(struct Backend, cfg));
  printf("\"Backend.kernels\": %zu,\n", offsetof(struct Backend, kernels));
  printf("\"Backend.impl\": %zu\n", offsetof(struct Backend, impl));
  printf("}\n");
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as td:
        c = os.path.join(td, "layout.c")
        open(c, "w").write(src)
        exe = os.path.join(td, "layout")
        subprocess.run(["gcc", "-std=c11", f"-I{a.ref}/src/include", f"-I{a.ref}/src/backend", c, "-o", exe],
                       check=True)
        txt = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    layout = json.loads(txt)
    with open(os.path.join(HERE, "abi_layout.json"), "w") as f:
        json.dump(layout, f, indent=1, sort_keys=True)
    print("wrote", len(out), "arrays and", len(layout), "layout entries")


if __name__ == "__main__":
    main()
