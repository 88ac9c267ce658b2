"""ctypes bindings for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke(), bench.py's CPU legs and the GPU
comparison script beside it (ref_cuda_compare.py) import this module.  It loads

* ``oracle/liboracle.so`` -- the plain-C restatement of the reference hot path
  (gb_oracle.c), and
* ``oracle/_ref/libref.so`` -- the reference's own CPU kernels compiled
  unchanged from the reference tree (oracle/Makefile), when it was built.

All array arguments are numpy arrays (C-contiguous); helpers return numpy.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
Q4K_BYTES, Q6K_BYTES, Q80_BYTES = 144, 210, 34
Q5K_BYTES, F16_BYTES = 176, 64   # F16 in "blocks" of 32 halves
DT_Q8_0, DT_Q4_K, DT_Q6_K, DT_F32 = 2, 4, 5, 0
DT_F16, DT_Q5_K = 1, 13   # Q5_K: GGML's type number (the reference's DataType has no Q5_K)

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and _ref/libref.so when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        vp, i, sz, u64 = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64
        for name in ("gbo_matvec_q4k", "gbo_matvec_q6k", "gbo_matvec_q8_0", "gbo_matvec_q5k", "gbo_matvec_f16"):
            getattr(L, name).argtypes = [vp, i, i, sz, vp, vp]
            getattr(L, name).restype = i
        for name in ("gbo_dequant_q4k", "gbo_dequant_q6k", "gbo_dequant_q8_0", "gbo_dequant_q5k", "gbo_dequant_f16"):
            getattr(L, name).argtypes = [vp, sz, vp]
            getattr(L, name).restype = None
        for name in ("gbo_synth_q4k", "gbo_synth_q6k", "gbo_synth_q8_0", "gbo_synth_q5k", "gbo_synth_f16"):
            getattr(L, name).argtypes = [vp, sz, u64, u64]
            getattr(L, name).restype = None
        L.gbo_synth_normal.argtypes = [vp, sz, u64, u64]
        L.gbo_rand64.argtypes = [u64, u64, u64]
        L.gbo_rand64.restype = u64
        L.gbo_f16_to_f32.argtypes = [C.c_uint16]
        L.gbo_f16_to_f32.restype = C.c_float
        L.gbo_f32_to_f16.argtypes = [C.c_float]
        L.gbo_f32_to_f16.restype = C.c_uint16
        L.gbo_rope.argtypes = [vp, vp, i, i, i, i, C.c_float]
        L.gbo_kv_append.argtypes = [vp, vp, vp, vp, i, i, i, i]
        L.gbo_attention.argtypes = [vp, vp, vp, i, i, i, i, i, vp]
        L.gbo_rmsnorm.argtypes = [vp, vp, vp, i, C.c_float]
        L.gbo_silu_mul.argtypes = [vp, vp, i]
        L.gbo_argmax.argtypes = [vp, i]
        L.gbo_argmax.restype = i
        L.gbo_layer_decode.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, C.c_float, C.c_float]
        L.gbo_layer_decode.restype = i
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libref.so"))


def _bind_harness(R) -> None:
    vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
    R.ref_set_threads.argtypes = [i]
    R.ref_matvec.argtypes = [i, vp, i, i, sz, vp, vp]
    R.ref_matvec.restype = i
    R.ref_dequant.argtypes = [i, vp, i, vp]
    R.ref_dequant.restype = i
    R.ref_attention_step.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, vp]
    R.ref_attention_step.restype = i
    R.ref_model_create.argtypes = [vp]
    R.ref_model_create.restype = vp
    R.ref_model_kv.argtypes = [vp, i, i]
    R.ref_model_kv.restype = C.POINTER(C.c_float)
    R.ref_model_forward.argtypes = [vp, i, i, vp]
    R.ref_model_forward.restype = i
    R.ref_model_forward_n.argtypes = [vp, vp, i, i, vp]
    R.ref_model_forward_n.restype = i
    R.ref_model_destroy.argtypes = [vp]


_dropin = None


def dropin_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libref_dropin.so"))


def dropin() -> C.CDLL:
    """The reference engine compiled with -DUSE_CUDA=1 against
    libguanaco_b200.so (oracle/_ref/libref_dropin.so): its forward() runs the
    drop-in cuda_transformer_layer_gpu once ref_model_to_gpu has moved a
    model's layers to the device.  Loaded privately (RTLD_LOCAL), so its copy
    of the reference symbols never mixes with libref.so's."""
    global _dropin
    if _dropin is None:
        path = os.path.join(HERE, "_ref", "libref_dropin.so")
        if not os.path.exists(path):
            raise FileNotFoundError("oracle/_ref/libref_dropin.so not built (reference tree absent)")
        R = C.CDLL(path, mode=os.RTLD_LOCAL)
        _bind_harness(R)
        R.ref_model_to_gpu.argtypes = [C.c_void_p, C.c_int]
        R.ref_model_to_gpu.restype = C.c_int
        _dropin = R
    return _dropin


def ref() -> C.CDLL:
    """The reference's own CPU kernels (oracle/_ref/libref.so)."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref.so")
        if not os.path.exists(path):
            raise FileNotFoundError("oracle/_ref/libref.so not built (reference tree absent)")
        R = C.CDLL(path, mode=os.RTLD_LOCAL)
        vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
        R.ref_set_threads.argtypes = [i]
        R.ref_matvec.argtypes = [i, vp, i, i, sz, vp, vp]
        R.ref_matvec.restype = i
        R.ref_dequant.argtypes = [i, vp, i, vp]
        R.ref_dequant.restype = i
        R.ref_attention_step.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, vp]
        R.ref_attention_step.restype = i
        R.ref_model_create.argtypes = [vp]
        R.ref_model_create.restype = vp
        R.ref_model_kv.argtypes = [vp, i, i]
        R.ref_model_kv.restype = C.POINTER(C.c_float)
        R.ref_model_forward.argtypes = [vp, i, i, vp]
        R.ref_model_forward.restype = i
        R.ref_model_destroy.argtypes = [vp]
        R.ref_model_forward_n.argtypes = [vp, vp, i, i, vp]
        R.ref_model_forward_n.restype = i
        _ref = R
    return _ref


# ---------------------------------------------------------------- synthesis
def block_bytes(dtype: int) -> int:
    return {DT_Q4_K: Q4K_BYTES, DT_Q6_K: Q6K_BYTES, DT_Q8_0: Q80_BYTES, DT_Q5_K: Q5K_BYTES, DT_F16: F16_BYTES}[dtype]


def weights_per_block(dtype: int) -> int:
    return 32 if dtype in (DT_Q8_0, DT_F16) else 256


def synth_blocks(dtype: int, rows: int, cols: int, seed: int, stream: int) -> np.ndarray:
    nb = rows * (cols // weights_per_block(dtype))
    out = np.empty(nb * block_bytes(dtype), dtype=np.uint8)
    fn = {DT_Q4_K: "gbo_synth_q4k", DT_Q6_K: "gbo_synth_q6k", DT_Q8_0: "gbo_synth_q8_0", DT_Q5_K: "gbo_synth_q5k",
          DT_F16: "gbo_synth_f16"}[dtype]
    getattr(lib(), fn)(_p(out), nb, seed, stream)
    return out


def synth_normal(n: int, seed: int, stream: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().gbo_synth_normal(_p(out), n, seed, stream)
    return out


# ---------------------------------------------------------------- compute
def matvec(dtype: int, W: np.ndarray, rows: int, cols: int, x: np.ndarray, byte_size: int = 0):
    y = np.zeros(rows, dtype=np.float32)
    fn = {DT_Q4_K: "gbo_matvec_q4k", DT_Q6_K: "gbo_matvec_q6k", DT_Q8_0: "gbo_matvec_q8_0", DT_Q5_K: "gbo_matvec_q5k",
          DT_F16: "gbo_matvec_f16"}[dtype]
    rc = getattr(lib(), fn)(_p(W), rows, cols, byte_size, _p(x), _p(y))
    return rc, y


def dequant(dtype: int, blocks: np.ndarray) -> np.ndarray:
    nb = blocks.size // block_bytes(dtype)
    out = np.empty(nb * weights_per_block(dtype), dtype=np.float32)
    fn = {DT_Q4_K: "gbo_dequant_q4k", DT_Q6_K: "gbo_dequant_q6k", DT_Q8_0: "gbo_dequant_q8_0", DT_Q5_K: "gbo_dequant_q5k",
          DT_F16: "gbo_dequant_f16"}[dtype]
    getattr(lib(), fn)(_p(blocks), nb, _p(out))
    return out


def attention_step(q, k, v, k_cache, v_cache, n_heads, n_kv, hd, max_seq, pos, theta=500000.0):
    """RoPE(q,k) -> append(k,v) -> attention, on copies; returns (out, kc, vc)."""
    q, k = q.copy(), k.copy()
    kc, vc = k_cache.copy(), v_cache.copy()
    L = lib()
    L.gbo_rope(_p(q), _p(k), n_heads, n_kv, hd, pos, theta)
    L.gbo_kv_append(_p(kc), _p(vc), _p(k), _p(v), n_kv, hd, max_seq, pos)
    out = np.empty(n_heads * hd, dtype=np.float32)
    L.gbo_attention(_p(q), _p(kc), _p(vc), n_heads, n_kv, hd, max_seq, pos, _p(out))
    return out, kc, vc


def rmsnorm(x, w, eps):
    out = np.empty_like(x)
    lib().gbo_rmsnorm(_p(x), _p(w) if w is not None else None, _p(out), x.size, eps)
    return out


def silu_mul(gate, up):
    g = gate.copy()
    lib().gbo_silu_mul(_p(g), _p(up), g.size)
    return g


def argmax(logits) -> int:
    return int(lib().gbo_argmax(_p(logits), logits.size))


class _Layer(C.Structure):
    _fields_ = [("w", C.c_void_p * 7), ("rows", C.c_int * 7), ("cols", C.c_int * 7),
                ("dtype", C.c_int * 7), ("rms_att", C.c_void_p), ("rms_ffn", C.c_void_p)]


def layer_decode(weights, dtypes, shapes, rms_att, rms_ffn, hidden, k_cache, v_cache,
                 H, n_heads, n_kv, hd, ff, max_seq, pos, eps=1e-6, theta=500000.0):
    """One decode layer on copies of hidden / caches; returns (hidden, kc, vc)."""
    Ls = _Layer()
    for i in range(7):
        Ls.w[i] = weights[i].ctypes.data
        Ls.rows[i], Ls.cols[i] = shapes[i]
        Ls.dtype[i] = dtypes[i]
    Ls.rms_att = rms_att.ctypes.data
    Ls.rms_ffn = rms_ffn.ctypes.data
    h = hidden.copy()
    kc, vc = k_cache.copy(), v_cache.copy()
    rc = lib().gbo_layer_decode(C.byref(Ls), _p(h), _p(kc), _p(vc), H, n_heads, n_kv, hd, ff,
                                max_seq, pos, eps, theta)
    if rc != 0:
        raise RuntimeError(f"gbo_layer_decode rc={rc}")
    return h, kc, vc


# ---------------------------------------------------------------- reference
def ref_matvec(dtype, W, rows, cols, x, byte_size=0):
    y = np.zeros(rows, dtype=np.float32)
    rc = ref().ref_matvec(dtype, _p(W), rows, cols, byte_size, _p(x), _p(y))
    return rc, y


def ref_dequant(dtype, blocks):
    nb = blocks.size // block_bytes(dtype)
    out = np.empty(nb * weights_per_block(dtype), dtype=np.float32)
    rc = ref().ref_dequant(dtype, _p(blocks), nb, _p(out))
    if rc != 0:
        raise RuntimeError("ref_dequant unsupported dtype")
    return out


def ref_attention_step(q, k, v, k_cache, v_cache, n_heads, n_kv, hd, max_seq, pos):
    q, k = q.copy(), k.copy()
    kc, vc = k_cache.copy(), v_cache.copy()
    out = np.empty(n_heads * hd, dtype=np.float32)
    rc = ref().ref_attention_step(_p(q), _p(k), _p(v), _p(kc), _p(vc), n_heads, n_kv, hd,
                                  max_seq, pos, _p(out))
    if rc != 0:
        raise RuntimeError(f"ref_attention_step rc={rc}")
    return out, kc, vc


class _ModelDesc(C.Structure):
    _fields_ = [("H", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int), ("hd", C.c_int),
                ("ff", C.c_int), ("vocab", C.c_int), ("n_layers", C.c_int), ("max_seq", C.c_int),
                ("w", C.POINTER(C.c_void_p)), ("w_dtype", C.POINTER(C.c_int)),
                ("rms_att", C.POINTER(C.c_void_p)), ("rms_ffn", C.POINTER(C.c_void_p)),
                ("embedding", C.c_void_p), ("emb_dtype", C.c_int),
                ("rms_final", C.c_void_p),
                ("lm_head", C.c_void_p), ("lm_dtype", C.c_int)]


class RefModel:
    """The reference forward() (engine.c:559-594) over caller-owned weights.
    lib: the harness to run it in (ref() by default; dropin() for the engine
    built with -DUSE_CUDA=1, see to_gpu)."""

    def __init__(self, model, lib=None):
        self._L = lib or ref()
        m = model
        n = m.n_layers
        self._keep = m
        self._w = (C.c_void_p * (7 * n))(*[w.ctypes.data for L in m.layers for w in L.w])
        self._dt = (C.c_int * (7 * n))(*[d for L in m.layers for d in L.dtypes])
        self._ra = (C.c_void_p * n)(*[L.rms_att.ctypes.data for L in m.layers])
        self._rf = (C.c_void_p * n)(*[L.rms_ffn.ctypes.data for L in m.layers])
        d = _ModelDesc(m.H, m.n_heads, m.n_kv, m.hd, m.ff, m.vocab, n, m.max_seq,
                       C.cast(self._w, C.POINTER(C.c_void_p)), C.cast(self._dt, C.POINTER(C.c_int)),
                       C.cast(self._ra, C.POINTER(C.c_void_p)), C.cast(self._rf, C.POINTER(C.c_void_p)),
                       m.embedding.ctypes.data, m.emb_dtype, m.rms_final.ctypes.data,
                       m.lm_head.ctypes.data, m.lm_dtype)
        self._d = d
        self.h = self._L.ref_model_create(C.byref(d))
        if not self.h:
            raise MemoryError("ref_model_create failed")

    def kv(self, layer: int, which_v: int, count: int) -> np.ndarray:
        p = self._L.ref_model_kv(self.h, layer, which_v)
        return np.ctypeslib.as_array(p, shape=(count,))

    def forward(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self._keep.vocab, dtype=np.float32)
        rc = self._L.ref_model_forward(self.h, token, pos, _p(logits))
        if rc != 0:
            raise RuntimeError("ref forward failed")
        return logits

    def forward_tokens(self, tokens, pos: int) -> np.ndarray:
        """forward() over a prompt of T = len(tokens) tokens at positions pos ..
        pos + T - 1 (the reference's CPU prefill): logits of the last."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self._keep.vocab, dtype=np.float32)
        rc = self._L.ref_model_forward_n(self.h, _p(t), t.size, pos, _p(logits))
        if rc != 0:
            raise RuntimeError("ref forward failed")
        return logits

    def to_gpu(self, threads: int) -> None:
        """Engine CUDA set-up (dropin() harness only): device copies of the
        layer matrices and the kernel table of backend_create(AUTO)."""
        rc = self._L.ref_model_to_gpu(self.h, threads)
        if rc != 0:
            raise RuntimeError(f"ref_model_to_gpu rc={rc}")

    def close(self):
        if self.h:
            self._L.ref_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
