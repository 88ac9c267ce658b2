"""Argument handling of the three vtable matvec slots that backend_cuda_create
installs (the engine calls them through linear_dispatch, engine.c:123-146),
case by case against the reference CPU kernels compiled into oracle/_ref
(quant_matvec_q4_k.c:142-158, quant_matvec_q6_k.c:43-58,
quant_matvec_q8_0.c:41-56): -1 for a NULL pointer, a wrong dtype or ndim, -2
for columns that are not a multiple of the block width, -3 for a known byte
size that is too small, and 0 for an empty matrix (no rows: nothing written;
no columns: every output 0).  Each case returns before any device work, so
these run without a GPU."""
import ctypes as C

import numpy as np
import pytest

SLOTS = {4: "q4k", 5: "q6k", 2: "q8_0"}
WIDTH = {4: 256, 5: 256, 2: 32}


@pytest.fixture(scope="module")
def fns(gb, oracle):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    ours, ref = {}, {}
    R = oracle.ref()
    for dt, name in SLOTS.items():
        for lib, table, sym in ((gb.lib(), ours, f"gb_backend_matvec_{name}_f32"), (R, ref, f"matvec_{name}_f32")):
            f = getattr(lib, sym)
            f.argtypes = [C.POINTER(gb.Tensor), C.c_void_p, C.c_void_p]
            f.restype = C.c_int
            table[dt] = f
    return ours, ref


def _call(f, t, x, y):
    return f(C.byref(t) if t is not None else None, x.ctypes.data if x is not None else None,
             y.ctypes.data if y is not None else None)


def _cases(gb, oracle, dt):
    """(name, tensor, x, y, expected code) with buffers kept alive."""
    w = WIDTH[dt]
    rows, cols = 8, 2 * w
    W = oracle.synth_blocks(dt, rows, cols, 17, 1)
    x = oracle.synth_normal(cols, 17, 2)
    other = {4: 5, 5: 2, 2: 4}[dt]

    def y():
        return np.full(rows, np.nan, np.float32)

    short = gb.make_tensor(dt, W, rows, cols, byte_size=W.nbytes - 1)
    wrong_dtype = gb.make_tensor(dt, W, rows, cols)
    wrong_dtype.dtype = other
    one_dim = gb.make_tensor(dt, W, rows, cols)
    one_dim.ndim = 1
    ragged = gb.make_tensor(dt, W, rows, cols + w // 2, byte_size=0)
    no_rows = gb.make_tensor(dt, W, 0, cols)
    no_cols = gb.make_tensor(dt, W, rows, 0)
    ok = gb.make_tensor(dt, W, rows, cols)
    return [
        ("null tensor", None, x, y(), -1),
        ("null x", ok, None, y(), -1),
        ("null y", ok, x, None, -1),
        ("wrong dtype", wrong_dtype, x, y(), -1),
        ("ndim 1", one_dim, x, y(), -1),
        ("ragged columns", ragged, x, y(), -2),
        ("byte size one short", short, x, y(), -3),
        ("no rows", no_rows, x, y(), 0),
        ("no columns", no_cols, x, y(), 0),
    ], W


@pytest.mark.parametrize("dt", list(SLOTS))
def test_vtable_argument_codes_match_reference(gb, oracle, fns, dt):
    ours, ref = fns
    cases, _keep = _cases(gb, oracle, dt)
    for name, t, x, y, want in cases:
        y_ours = None if y is None else y.copy()
        y_ref = None if y is None else y.copy()
        got = _call(ours[dt], t, x, y_ours)
        exp = _call(ref[dt], t, x, y_ref)
        assert exp == want, (name, exp)
        assert got == exp, (name, got, exp)
        if y is not None:
            # same outputs: untouched on an error or with no rows, zeros with no columns
            assert np.array_equal(np.isnan(y_ours), np.isnan(y_ref)), name
            assert np.array_equal(np.nan_to_num(y_ours), np.nan_to_num(y_ref)), name


def test_cuda_backend_absent_without_a_device(gb):
    """backend_cuda_create returns NULL when no CUDA device is present, so the
    reference's AUTO selection (backend.c:15-35) falls back to its CPU
    backend."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    cfg = gb.BackendConfig(1, 1, 0, 0)
    assert not gb.lib().backend_cuda_create(C.byref(cfg))
