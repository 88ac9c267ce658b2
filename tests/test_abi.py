"""CPU: the C-ABI library loads, exports every function include/*.h declares,
and the mirrored reference structs have the reference's layout."""
import ctypes as C
import json
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("guanaco_b200.h", "guanaco_backend_abi.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M):
            if m.group(1) not in ("if", "while", "sizeof", "return", "typedef"):
                names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(gb):
    names = declared_functions()
    assert {"cuda_transformer_layer_gpu", "cuda_upload_weight", "backend_cuda_create",
            "gb_matvec", "gb_attention_decode", "gb_model_decode"} <= names
    L = gb.lib()
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding knows every declared symbol too
    assert names <= set(gb.SIGNATURES), sorted(names - set(gb.SIGNATURES))


def test_library_is_the_in_tree_build(gb):
    assert os.path.realpath(gb.LIB_PATH).startswith(ROOT)
    assert gb.lib().gb_version().decode().startswith("guanaco_b200")


def test_struct_layout_matches_reference(gb):
    ref = json.load(open(os.path.join(ROOT, "tests", "golden", "abi_layout.json")))
    assert C.sizeof(gb.Tensor) == ref["sizeof.Tensor"]
    for f in ("data", "shape", "stride", "ndim", "dtype", "ggml_type", "byte_size", "device_residency", "d_data"):
        assert getattr(gb.Tensor, f).offset == ref["Tensor." + f], f
    assert C.sizeof(gb.BackendConfig) == ref["sizeof.BackendConfig"]
    for f in ("kind", "threads", "device_id", "n_gpu_layers"):
        assert getattr(gb.BackendConfig, f).offset == ref["BackendConfig." + f]
    assert C.sizeof(gb.KernelVTable) == ref["sizeof.KernelVTable"]
    for f in ("gemm_f32", "elemwise_mul", "matvec_q4k_f32", "matvec_q6k_f32", "matvec_q8_0_f32"):
        assert getattr(gb.KernelVTable, f).offset == ref["KernelVTable." + f]
    assert C.sizeof(gb.Backend) == ref["sizeof.Backend"]
    for f in ("cfg", "kernels", "impl"):
        assert getattr(gb.Backend, f).offset == ref["Backend." + f]


def test_c_header_layout_matches_reference(tmp_path):
    """Compile include/guanaco_backend_abi.h (the stand-alone mirror) and
    compare its offsets with the reference's."""
    import subprocess
    ref = json.load(open(os.path.join(ROOT, "tests", "golden", "abi_layout.json")))
    src = tmp_path / "l.c"
    src.write_text(r'''
#include <stdio.h>
#include <stddef.h>
#include "guanaco_backend_abi.h"
int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(Tensor), offsetof(Tensor, byte_size),
 offsetof(Tensor, d_data), sizeof(BackendConfig), sizeof(KernelVTable), offsetof(KernelVTable, matvec_q8_0_f32),
 sizeof(struct Backend), offsetof(struct Backend, impl)); return 0;}''')
    exe = tmp_path / "l"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT}/include", str(src), "-o", str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()))
    want = [ref["sizeof.Tensor"], ref["Tensor.byte_size"], ref["Tensor.d_data"], ref["sizeof.BackendConfig"],
            ref["sizeof.KernelVTable"], ref["KernelVTable.matvec_q8_0_f32"], ref["sizeof.Backend"], ref["Backend.impl"]]
    assert got == want


def test_no_cpu_fallback_when_library_missing(gb, monkeypatch):
    import guanaco_b200 as G
    monkeypatch.setattr(G, "_lib", None)
    monkeypatch.setattr(G, "LIB_PATH", "/nonexistent/libguanaco_b200.so")
    import pytest
    with pytest.raises(RuntimeError):
        G.lib()


def test_product_does_not_touch_the_oracle():
    """The shipped library and package never reference oracle code."""
    pkg = os.path.join(ROOT, "guanaco_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".c", ".h", ".cuh")):
                txt = open(os.path.join(dirpath, f)).read()
                assert "gbo_" not in txt and "oracle" not in txt.lower().replace("oracle.", ""), f


def test_gemm_split_bytes_without_a_gpu(gb):
    """gb_gemm_split_bytes is host arithmetic: token rows rounded up to the
    256-row pitch of the column-group-major split, 2 bytes per element."""
    assert gb.gemm_split_bytes(300, 1024) == 512 * 1024 * 2
    assert gb.gemm_split_bytes(256, 4096) == 256 * 4096 * 2
    assert gb.gemm_split_bytes(1, 32) == 256 * 32 * 2
    assert gb.gemm_split_bytes(0, 4096) == 0
    assert gb.gemm_split_bytes(16, -1) == 0
