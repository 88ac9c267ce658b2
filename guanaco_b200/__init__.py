"""guanaco_b200 -- B200 (sm_100a) decode hot path for the Guanaco GGUF engine.

The product is ``lib/libguanaco_b200.so`` (CUDA kernels + C11 host code behind
the C ABI in ``include/guanaco_b200.h`` and ``include/guanaco_backend_abi.h``).
This module is a thin ctypes binding over that ABI for Python callers, the
tests and the benchmark.  There is no CPU fallback: if the shared library is
missing or fails to load, :func:`lib` raises.

Device buffers are passed as raw pointers; the helpers accept torch CUDA
tensors (torch is only the device-memory / stream plumbing here).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libguanaco_b200.so")

DT_F32, DT_Q8_0, DT_Q4_K, DT_Q6_K = 0, 2, 4, 5
DT_F16, DT_Q5_K = 1, 13   # Q5_K: GGML's type number (no reference DataType)
BLOCK_BYTES = {DT_Q4_K: 144, DT_Q6_K: 210, DT_Q8_0: 34, DT_Q5_K: 176, DT_F16: 64}   # F16: blocks of 32 halves
BLOCK_WIDTH = {DT_Q4_K: 256, DT_Q6_K: 256, DT_Q8_0: 32, DT_Q5_K: 256, DT_F16: 32}
WQ, WK, WV, WO, WGATE, WUP, WDOWN = range(7)

GB_OK, GB_EINVAL, GB_ESHAPE, GB_ESIZE, GB_EPOS, GB_ECUDA, GB_ENOMEM, GB_ETIMEOUT, GB_ELIMIT = \
    0, -1, -2, -3, -4, -5, -6, -7, -8

_lib = None


class GBError(RuntimeError):
    def __init__(self, fn: str, rc: int):
        super().__init__(f"{fn} failed with code {rc}")
        self.rc = rc


def build() -> None:
    """Compile the CUDA library in-tree (nvcc for sm_100a; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


# ------------------------------------------------------------- ABI structs
class Tensor(C.Structure):
    """The reference Tensor (src/include/types.h:51-62), field for field."""
    _fields_ = [("data", C.c_void_p), ("shape", C.c_int * 4), ("stride", C.c_int * 4),
                ("ndim", C.c_int), ("dtype", C.c_int), ("ggml_type", C.c_uint32),
                ("byte_size", C.c_size_t), ("device_residency", C.c_int), ("d_data", C.c_void_p)]


class BackendConfig(C.Structure):
    """src/include/backend.h:41-46."""
    _fields_ = [("kind", C.c_int), ("threads", C.c_int), ("device_id", C.c_int), ("n_gpu_layers", C.c_int)]


_MATVEC_FN = C.CFUNCTYPE(C.c_int, C.POINTER(Tensor), C.c_void_p, C.c_void_p)


class KernelVTable(C.Structure):
    """src/include/backend.h:21-39 (glue slots kept opaque)."""
    _fields_ = [("gemm_f32", C.c_void_p), ("gemm_f32_nn", C.c_void_p), ("rmsnorm", C.c_void_p),
                ("softmax_inplace", C.c_void_p), ("silu_inplace", C.c_void_p), ("rope", C.c_void_p),
                ("residual_add", C.c_void_p), ("elemwise_mul", C.c_void_p),
                ("matvec_q4k_f32", _MATVEC_FN), ("matvec_q6k_f32", _MATVEC_FN),
                ("matvec_q8_0_f32", _MATVEC_FN)]


class Backend(C.Structure):
    """struct Backend (src/backend/backend_internal.h:7-11)."""
    _fields_ = [("cfg", BackendConfig), ("kernels", KernelVTable), ("impl", C.c_void_p)]


class ModelConfig(C.Structure):
    _fields_ = [("hidden_dim", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("n_layers", C.c_int), ("ff_dim", C.c_int), ("vocab_size", C.c_int), ("max_seq", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float)]


# Every symbol the C headers declare, with its ctypes signature.
_vp, _i, _sz, _u64, _f = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64, C.c_float
SIGNATURES = {
    # drop-in symbols
    "cuda_upload_weight": (_vp, [_vp, _sz]),
    "cuda_matvec_q4k_f32_impl": (_i, [_vp, _vp, _vp, _i, _i]),
    "cuda_transformer_layer_gpu": (_i, [_vp, _i, _i, _i] * 7 + [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i]),
    "cuda_finish_layer": (None, []),
    "cuda_sync_kv_cache": (None, [_i, _i, _i, _i, _i, _vp, _vp, _i, _i]),
    "cuda_get_temperature": (_i, []),
    "backend_cuda_create": (C.POINTER(Backend), [C.POINTER(BackendConfig)]),
    "backend_cuda_destroy": (None, [C.POINTER(Backend)]),
    "gb_backend_matvec_q4k_f32": (_i, [C.POINTER(Tensor), _vp, _vp]),
    "gb_backend_matvec_q6k_f32": (_i, [C.POINTER(Tensor), _vp, _vp]),
    "gb_backend_matvec_q8_0_f32": (_i, [C.POINTER(Tensor), _vp, _vp]),
    # native API
    "gb_version": (C.c_char_p, []),
    "gb_device_sm_count": (_i, []),
    "gb_matvec": (_i, [_i, _vp, _i, _i, _vp, _vp, _vp, _vp]),
    "gb_matvec_group": (_i, [_i, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "gb_matvec_host": (_i, [_i, _vp, _i, _i, _vp, _vp]),
    "gb_vtable_cache_clear": (_i, []),
    "gb_device_error": (_i, [_i]),
    "gb_gemm": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "gb_gemm_error": (_i, [_i]),
    "gb_gemm_split_bytes": (_sz, [_i, _i]),
    "gb_gemm_split": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "gb_gemm_presplit": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "gb_prefill_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "gb_prefill_attention_error": (_i, [_i]),
    "gb_dequant": (_i, [_i, _vp, _sz, _vp, _vp]),
    "gb_synth_blocks": (_i, [_i, _vp, _sz, _u64, _u64, _vp]),
    "gb_synth_normal": (_i, [_vp, _sz, _u64, _u64, _vp]),
    "gb_fill_f32": (_i, [_vp, _sz, _f, _vp]),
    "gb_rope_table": (_i, [_vp, _i, _i, _f, _vp]),
    "gb_attn_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "gb_attention_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "gb_attention_decode_static": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "gb_attention_static_error": (_i, [_i]),
    "gb_rmsnorm": (_i, [_vp, _vp, _vp, _i, _f, _vp]),
    "gb_silu_mul": (_i, [_vp, _vp, _i, _vp]),
    "gb_argmax": (_i, [_vp, _i, _vp, _vp]),
    "gb_model_create": (_vp, [C.POINTER(ModelConfig)]),
    "gb_model_create_tp": (_vp, [C.POINTER(ModelConfig), _i, _i]),
    "gb_model_comm_handle": (_i, [_vp, _vp]),
    "gb_model_comm_open": (_i, [_vp, _vp]),
    "gb_model_tp_info": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "gb_model_destroy": (None, [_vp]),
    "gb_model_set_matrix": (_i, [_vp, _i, _i, _i, _vp]),
    "gb_model_set_norms": (_i, [_vp, _i, _vp, _vp]),
    "gb_model_set_head": (_i, [_vp, _i, _vp, _vp, _i, _vp]),
    "gb_model_synthesize": (_i, [_vp, _u64]),
    "gb_model_k_cache": (_vp, [_vp, _i]),
    "gb_model_v_cache": (_vp, [_vp, _i]),
    "gb_model_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "gb_model_decode_host": (_i, [_vp, _i, _i, _vp, _vp]),
    "gb_model_prefill": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "gb_model_prefill_host": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "gb_model_step_bytes": (C.c_double, [_vp, _i]),
    "gb_model_generate": (_i, [_vp, _vp, _vp, _i, _vp, _vp]),
    "gb_model_fill_kv": (_i, [_vp, _i, _u64]),
    "gb_model_error": (_i, [_vp]),
    "gb_model_launches_per_step": (_i, [_vp]),
}


def lib() -> C.CDLL:
    """Load libguanaco_b200.so; raises if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run guanaco_b200.build() (nvcc, sm_100a)")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream


def check(fn: str, rc: int) -> None:
    if rc != 0:
        raise GBError(fn, rc)


# ------------------------------------------------------------- native API
def matvec(dtype, W, rows, cols, x, y, residual=None, stream=None) -> None:
    check("gb_matvec", lib().gb_matvec(dtype, _ptr(W), rows, cols, _ptr(x), _ptr(y), _ptr(residual),
                                        _stream(stream)))


def matvec_group(dtypes, Ws, rows, cols, x, ys, stream=None) -> None:
    """ys[i] = Ws[i] . x for up to three matrices sharing x (one launch when
    their formats allow it)."""
    n = len(Ws)
    dt = (C.c_int * n)(*dtypes)
    wp = (C.c_void_p * n)(*[_ptr(w) for w in Ws])
    rw = (C.c_int * n)(*rows)
    yp = (C.c_void_p * n)(*[_ptr(v) for v in ys])
    check("gb_matvec_group", lib().gb_matvec_group(n, dt, wp, rw, cols, _ptr(x), yp, _stream(stream)))


def gemm(dtype, W, X, Y, N, K, T, R=None, stream=None) -> None:
    """Y[t][n] = sum_k X[t][k] W[n][k] (+ R[t][n]) on the tensor cores (prefill)."""
    check("gb_gemm", lib().gb_gemm(dtype, _ptr(W), _ptr(X), _ptr(Y), _ptr(R), N, K, T, _stream(stream)))


def gemm_split(X, T, K, hi, lo, inv, stream=None) -> None:
    """Split X [T][K] once for fp16-operand GEMMs (hi / lo: gemm_split_bytes each)."""
    check("gb_gemm_split", lib().gb_gemm_split(_ptr(X), T, K, _ptr(hi), _ptr(lo), _ptr(inv), _stream(stream)))


def gemm_split_bytes(T, K) -> int:
    return int(lib().gb_gemm_split_bytes(T, K))


def gemm_presplit(dtype, W, hi, lo, inv, Y, N, K, T, R=None, stream=None) -> None:
    """gemm() on an X split by gemm_split()."""
    check("gb_gemm_presplit", lib().gb_gemm_presplit(dtype, _ptr(W), _ptr(hi), _ptr(lo), _ptr(inv), _ptr(Y), _ptr(R),
                                                     N, K, T, _stream(stream)))


def prefill_attention(q, k_cache, v_cache, out, n_tokens, pos, n_heads, n_kv, head_dim, max_seq,
                      stream=None) -> None:
    """Causal attention of n_tokens prompt rows (positions pos ..) over a layer's cache."""
    check("gb_prefill_attention", lib().gb_prefill_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                                             n_tokens, pos, n_heads, n_kv, head_dim, max_seq,
                                                             _stream(stream)))


def dequant(dtype, blocks, nblocks, out, stream=None) -> None:
    check("gb_dequant", lib().gb_dequant(dtype, _ptr(blocks), nblocks, _ptr(out), _stream(stream)))


def synth_blocks(dtype, buf, nblocks, seed, stream_id, stream=None) -> None:
    check("gb_synth_blocks", lib().gb_synth_blocks(dtype, _ptr(buf), nblocks, seed, stream_id, _stream(stream)))


def synth_normal(buf, n, seed, stream_id, stream=None) -> None:
    check("gb_synth_normal", lib().gb_synth_normal(_ptr(buf), n, seed, stream_id, _stream(stream)))


def rope_table(cs, max_seq, head_dim, theta=500000.0, stream=None) -> None:
    check("gb_rope_table", lib().gb_rope_table(_ptr(cs), max_seq, head_dim, theta, _stream(stream)))


def attn_workspace_bytes(n_heads, n_kv, head_dim, max_seq) -> int:
    return int(lib().gb_attn_workspace_bytes(n_heads, n_kv, head_dim, max_seq))


def attention_decode(q, k, v, k_cache, v_cache, rope_cs, d_pos, n_heads, n_kv, head_dim, max_seq, out, ws,
                     stream=None) -> None:
    check("gb_attention_decode", lib().gb_attention_decode(
        _ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(rope_cs), _ptr(d_pos),
        n_heads, n_kv, head_dim, max_seq, _ptr(out), _ptr(ws), _stream(stream)))


def attention_decode_static(q, k, v, k_cache, v_cache, rope_cs, d_pos, n_heads, n_kv, head_dim, max_seq, out,
                            stream=None) -> None:
    """gb_attention_decode with the library's static scratch (no workspace,
    no allocation); calls on one device must not overlap."""
    check("gb_attention_decode_static", lib().gb_attention_decode_static(
        _ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(rope_cs), _ptr(d_pos),
        n_heads, n_kv, head_dim, max_seq, _ptr(out), _stream(stream)))


def rmsnorm(x, w, out, n, eps, stream=None) -> None:
    check("gb_rmsnorm", lib().gb_rmsnorm(_ptr(x), _ptr(w), _ptr(out), n, eps, _stream(stream)))


def silu_mul(gate, up, n, stream=None) -> None:
    check("gb_silu_mul", lib().gb_silu_mul(_ptr(gate), _ptr(up), n, _stream(stream)))


def argmax(x, n, out, stream=None) -> None:
    check("gb_argmax", lib().gb_argmax(_ptr(x), n, _ptr(out), _stream(stream)))


def matrix_bytes(dtype, rows, cols) -> int:
    return rows * (cols // BLOCK_WIDTH[dtype]) * BLOCK_BYTES[dtype]


IPC_HANDLE_BYTES = 64


class DecodeModel:
    """Device-resident decode model (forward() at T = 1, greedy).  With
    tp_world > 1 this is rank tp_rank's tensor-parallel slice; call
    exchange_handles() (or comm_handle / comm_open) on every rank before
    decoding, and drive every rank through the same decode calls."""

    def __init__(self, hidden_dim, n_heads, n_kv_heads, n_layers, ff_dim, vocab_size, max_seq,
                 rms_eps=1e-6, rope_theta=500000.0, tp_rank=0, tp_world=1):
        self.cfg = ModelConfig(hidden_dim, n_heads, n_kv_heads, hidden_dim // n_heads, n_layers, ff_dim,
                               vocab_size, max_seq, rms_eps, rope_theta)
        self.tp_rank, self.tp_world = tp_rank, tp_world
        self.h = lib().gb_model_create_tp(C.byref(self.cfg), tp_rank, tp_world)
        if not self.h:
            raise GBError("gb_model_create_tp", GB_EINVAL)

    def comm_handle(self) -> bytes:
        buf = C.create_string_buffer(IPC_HANDLE_BYTES)
        check("gb_model_comm_handle", lib().gb_model_comm_handle(self.h, buf))
        return buf.raw

    def comm_open(self, handles) -> None:
        """handles: the world ranks' comm_handle() bytes, in rank order."""
        blob = b"".join(handles)
        if len(blob) != IPC_HANDLE_BYTES * self.tp_world:
            raise GBError("gb_model_comm_open", GB_EINVAL)
        buf = C.create_string_buffer(blob, len(blob))
        check("gb_model_comm_open", lib().gb_model_comm_open(self.h, buf))

    def exchange_handles(self, dist, group=None) -> None:
        """All-gather the ranks' handles with torch.distributed (any backend)
        and open the peers' exchange buffers."""
        out = [None] * self.tp_world
        dist.all_gather_object(out, self.comm_handle(), group=group)
        self.comm_open(out)

    def tp_info(self):
        r, w, off, n = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check("gb_model_tp_info", lib().gb_model_tp_info(self.h, C.byref(r), C.byref(w), C.byref(off), C.byref(n)))
        return r.value, w.value, off.value, n.value

    def synthesize(self, seed: int) -> None:
        check("gb_model_synthesize", lib().gb_model_synthesize(self.h, seed))

    def set_matrix(self, layer, which, dtype, W) -> None:
        check("gb_model_set_matrix", lib().gb_model_set_matrix(self.h, layer, which, dtype, _ptr(W)))

    def set_norms(self, layer, rms_att, rms_ffn) -> None:
        check("gb_model_set_norms", lib().gb_model_set_norms(self.h, layer, _ptr(rms_att), _ptr(rms_ffn)))

    def set_head(self, emb_dtype, emb, rms_final, lm_dtype, lm) -> None:
        check("gb_model_set_head", lib().gb_model_set_head(self.h, emb_dtype, _ptr(emb), _ptr(rms_final),
                                                           lm_dtype, _ptr(lm)))

    def k_cache(self, layer) -> int:
        return lib().gb_model_k_cache(self.h, layer)

    def v_cache(self, layer) -> int:
        return lib().gb_model_v_cache(self.h, layer)

    def decode(self, d_token, d_pos, d_logits, d_next, stream=None) -> None:
        check("gb_model_decode", lib().gb_model_decode(self.h, _ptr(d_token), _ptr(d_pos), _ptr(d_logits),
                                                       _ptr(d_next), _stream(stream)))

    def decode_host(self, token: int, pos: int, logits=None) -> int:
        nxt = C.c_int(0)
        ptr = None
        if logits is not None:
            ptr = logits.ctypes.data if hasattr(logits, "ctypes") else _ptr(logits)
        check("gb_model_decode_host", lib().gb_model_decode_host(self.h, token, pos, C.byref(nxt), ptr))
        return nxt.value

    def prefill(self, d_tokens, n_tokens: int, pos: int, d_logits, d_next, stream=None) -> None:
        """A prompt of n_tokens device tokens at positions pos ..: K / V cache
        rows written, last row's logits / argmax out (asynchronous)."""
        check("gb_model_prefill", lib().gb_model_prefill(self.h, _ptr(d_tokens), n_tokens, pos, _ptr(d_logits),
                                                         _ptr(d_next), _stream(stream)))

    def prefill_host(self, tokens, pos: int, logits=None) -> int:
        """Host prompt in, next token (and optionally the logits) out."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = C.c_int(0)
        ptr = None
        if logits is not None:
            ptr = logits.ctypes.data if hasattr(logits, "ctypes") else _ptr(logits)
        check("gb_model_prefill_host", lib().gb_model_prefill_host(self.h, t.ctypes.data, t.size, pos,
                                                                   C.byref(nxt), ptr))
        return nxt.value

    def generate(self, d_token, d_pos, n_steps, d_out=None, stream=None) -> None:
        check("gb_model_generate", lib().gb_model_generate(self.h, _ptr(d_token), _ptr(d_pos), n_steps,
                                                           _ptr(d_out), _stream(stream)))

    def fill_kv(self, n_pos: int, seed: int) -> None:
        check("gb_model_fill_kv", lib().gb_model_fill_kv(self.h, n_pos, seed))

    def error(self) -> int:
        return lib().gb_model_error(self.h)

    def launches_per_step(self) -> int:
        return lib().gb_model_launches_per_step(self.h)

    def step_bytes(self, pos: int) -> float:
        return float(lib().gb_model_step_bytes(self.h, pos))

    def close(self) -> None:
        if self.h:
            lib().gb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------- vtable mirror
class CudaBackend:
    """backend_cuda_create / backend_cuda_destroy and the three quantised
    vtable slots, called exactly as the engine calls them
    (src/engine/engine.c:123-146): ``slot(&W, x_host, y_host) -> int``."""

    def __init__(self, device_id=0, threads=1):
        self.cfg = BackendConfig(1, threads, device_id, 0)
        self.b = lib().backend_cuda_create(C.byref(self.cfg))
        if not self.b:
            raise GBError("backend_cuda_create", GB_EINVAL)
        self.kernels = self.b.contents.kernels

    def matvec(self, W: Tensor, x, y) -> int:
        fn = {DT_Q4_K: self.kernels.matvec_q4k_f32, DT_Q6_K: self.kernels.matvec_q6k_f32,
              DT_Q8_0: self.kernels.matvec_q8_0_f32}[W.dtype]
        return fn(C.byref(W), x.ctypes.data, y.ctypes.data)

    def close(self):
        if self.b:
            lib().backend_cuda_destroy(self.b)
            self.b = None


def make_tensor(dtype, host_array, rows, cols, byte_size=None, d_data=None) -> Tensor:
    """A 2-D quantised Tensor over host bytes (and optionally a device copy)."""
    t = Tensor()
    t.data = host_array.ctypes.data if host_array is not None else None
    t.shape[0], t.shape[1] = rows, cols
    t.stride[0], t.stride[1] = cols, 1
    t.ndim = 2
    t.dtype = dtype
    t.byte_size = host_array.nbytes if byte_size is None else byte_size
    t.device_residency = 1 if d_data else 0
    t.d_data = d_data
    return t
