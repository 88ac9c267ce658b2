"""Prefill GEMM on the tcgen05 tensor cores (gb_gemm): Y = X . W^T (+ R) for T
tokens at once, W fp32 or GGUF Q4_K / Q6_K / Q8_0 blocks dequantised on the
fly.  fp32-equivalent arithmetic (3xF16 with power-of-two row scales by
default, 3xTF32 with GB_GEMM_KIND=tf32; the tensor cores' accumulator is
restarted every 256 / 512 columns of K and the partial sums added in fp32),
so the result must match an fp64 product of the oracle's
dequantised weights (the reference's formulas) to a few 1e-6 relative L2
(bound 1e-5 at every K tested, up to 2048), far inside the 1e-3 bound."""
import numpy as np
import pytest

from tests.helpers import rel_l2, to_dev, from_dev

pytestmark = pytest.mark.gpu


def _run(gb, cuda, dt, Wdev, X, N, K, T, R=None):
    Xd = to_dev(cuda, X)
    Y = cuda.full((T, N), float("nan"), dtype=cuda.float32, device="cuda")
    Rd = to_dev(cuda, R) if R is not None else None
    gb.gemm(dt, Wdev, Xd, Y, N, K, T, R=Rd)
    cuda.cuda.synchronize()
    assert gb.lib().gb_gemm_error(1) == 0
    return from_dev(Y)


@pytest.mark.parametrize("N,K,T", [(128, 32, 16), (128, 256, 128), (200, 512, 130), (37, 96, 3), (300, 64, 257)])
def test_gemm_fp32_matches_fp64(gb, oracle, cuda, N, K, T):
    W = oracle.synth_normal(N * K, 3, N).reshape(N, K)
    X = oracle.synth_normal(T * K, 3, K + T).reshape(T, K)
    Y = _run(gb, cuda, 0, to_dev(cuda, W), X, N, K, T)
    ref = X.astype(np.float64) @ W.astype(np.float64).T
    assert np.all(np.isfinite(Y))
    assert rel_l2(Y, ref) <= 1e-5, rel_l2(Y, ref)


@pytest.mark.parametrize("dt", [4, 5, 2])
@pytest.mark.parametrize("N,K,T", [(128, 256, 1), (256, 1024, 128), (100, 512, 37), (260, 2048, 200),
                                   (256, 1024, 4096), (140, 4096, 1000)])
def test_gemm_quantised_matches_dequantised_product(gb, oracle, cuda, dt, N, K, T):
    W = oracle.synth_blocks(dt, N, K, 5, N + K)
    Wd = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    Wd[: W.size] = to_dev(cuda, W)
    X = oracle.synth_normal(T * K, 5, T).reshape(T, K)
    R = oracle.synth_normal(T * N, 5, 7).reshape(T, N)
    Y = _run(gb, cuda, dt, Wd, X, N, K, T, R=R)
    Wf = oracle.dequant(dt, W).reshape(N, K).astype(np.float64)
    ref = X.astype(np.float64) @ Wf.T + R
    assert rel_l2(Y, ref) <= 1e-5, rel_l2(Y, ref)
    # each row agrees with the reference's own matvec on that token
    for t in (0, T - 1):
        _, y = oracle.matvec(dt, W, N, K, X[t])
        assert rel_l2(Y[t] - R[t], y) <= 1e-5


def test_gemm_residual_in_place(gb, oracle, cuda):
    N, K, T = 256, 512, 40
    W = oracle.synth_blocks(4, N, K, 9, 1)
    Wd = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    Wd[: W.size] = to_dev(cuda, W)
    X = oracle.synth_normal(T * K, 9, 2).reshape(T, K)
    H = oracle.synth_normal(T * N, 9, 3).reshape(T, N)
    Hd = to_dev(cuda, H)
    gb.gemm(4, Wd, to_dev(cuda, X), Hd, N, K, T, R=Hd)
    cuda.cuda.synchronize()
    ref = X.astype(np.float64) @ oracle.dequant(4, W).reshape(N, K).astype(np.float64).T + H
    assert rel_l2(from_dev(Hd), ref) <= 1e-5


@pytest.mark.parametrize("dt", [4, 5])
def test_gemm_long_k_wide_tiles(gb, oracle, cuda, dt):
    """ffn_down's K = 14336 on the 256-token tiles (1280 rows x 4096 tokens: a
    grid of 10 x 16 CTAs, more than one per SM): 28 accumulator groups of 512
    columns; 64 sampled token rows against fp64."""
    N, K, T = 1280, 14336, 4096
    W = oracle.synth_blocks(dt, N, K, 21, 3)
    Wd = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    Wd[: W.size] = to_dev(cuda, W)
    X = oracle.synth_normal(T * K, 21, 4).reshape(T, K)
    Y = cuda.full((T, N), float("nan"), dtype=cuda.float32, device="cuda")
    gb.gemm(dt, Wd, to_dev(cuda, X), Y, N, K, T)
    cuda.cuda.synchronize()
    assert gb.lib().gb_gemm_error(1) == 0
    rows = np.random.RandomState(5).choice(T, 64, replace=False)
    Wf = oracle.dequant(dt, W).reshape(N, K).astype(np.float64)
    ref = X[rows].astype(np.float64) @ Wf.T
    got = from_dev(Y)[rows]
    assert np.all(np.isfinite(from_dev(Y)))
    assert rel_l2(got, ref) <= 1e-5, rel_l2(got, ref)


@pytest.mark.parametrize("N,K,T", [(256, 1024, 300), (128, 4096, 40)])
def test_gemm_presplit_equals_gemm(gb, oracle, cuda, N, K, T):
    """gb_gemm_split + gb_gemm_presplit (one split X for several GEMMs) give
    gb_gemm's result bit for bit, also for T not a multiple of the 256-row
    split pitch; the split X is reused by a second GEMM with a residual.
    Activations with a wide dynamic range (rows scaled by 2^-20 .. 2^12) keep
    the fp64 bound, since each token row has its own power-of-two scale."""
    W = oracle.synth_blocks(4, N, K, 9, N + K)
    X = oracle.synth_normal(T * K, 9, T).reshape(T, K)
    X *= np.exp2(np.linspace(-20, 12, T)).astype(np.float32)[:, None]
    Wd = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    Wd[: W.size] = cuda.from_numpy(W).cuda()
    ref_y = _run(gb, cuda, 4, Wd, X, N, K, T)
    sb = gb.gemm_split_bytes(T, K)
    assert sb == ((T + 255) // 256 * 256) * K * 2
    xh = cuda.empty(sb, dtype=cuda.uint8, device="cuda")
    xl = cuda.empty(sb, dtype=cuda.uint8, device="cuda")
    xi = cuda.empty(T, dtype=cuda.float32, device="cuda")
    gb.gemm_split(to_dev(cuda, X), T, K, xh, xl, xi)
    Y = cuda.full((T, N), float("nan"), dtype=cuda.float32, device="cuda")
    gb.gemm_presplit(4, Wd, xh, xl, xi, Y, N, K, T)
    R = oracle.synth_normal(T * N, 9, 7).reshape(T, N)
    Y2 = to_dev(cuda, R)
    gb.gemm_presplit(4, Wd, xh, xl, xi, Y2, N, K, T, R=Y2)
    cuda.cuda.synchronize()
    assert gb.lib().gb_gemm_error(1) == 0
    assert np.array_equal(from_dev(Y).view(np.uint32), ref_y.view(np.uint32))
    Wf = oracle.dequant(4, W).reshape(N, K).astype(np.float64)
    ref = X.astype(np.float64) @ Wf.T
    # relative to each token row's own magnitude
    err = np.linalg.norm(from_dev(Y) - ref, axis=1) / np.maximum(np.linalg.norm(ref, axis=1), 1e-300)
    assert err.max() <= 1e-5, err.max()
    assert rel_l2(from_dev(Y2), ref + R) <= 1e-5


def test_gemm_tf32_operands_in_a_subprocess():
    """The 3xTF32 form (GB_GEMM_KIND=tf32, read once per process) against the
    same fp64 bounds: the quantised GEMM cases, the long-K case and the
    model-level prefill parity of tests/test_gpu_prefill.py, run by pytest in
    a child process with the variable set."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, GB_GEMM_KIND="tf32")
    cmd = [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
           "tests/test_gpu_gemm.py::test_gemm_quantised_matches_dequantised_product",
           "tests/test_gpu_gemm.py::test_gemm_long_k_wide_tiles",
           "tests/test_gpu_gemm.py::test_gemm_fp32_matches_fp64",
           "tests/test_gpu_prefill.py::test_prefill_matches_reference_forward"]
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout, r.stdout[-2000:]
