"""Q5_K and F16 weights on the device: formats the reference loader sizes but
rejects (src/engine/loader.c:98,117,586-651), so parity is against the
oracle's restatement (GGML's block_q5_K layout; the reference's own fp16
mapping, engine.c:183-212), pinned on the CPU by tests/test_oracle_q5k_f16.py.

* device generators and gb_dequant bit-exact against the oracle;
* decode matvec (k_mv_plain) and prefill GEMM within 1e-5 relative L2 of an
  fp64 product of the dequantised rows (fp32 arithmetic; x exact in fp32);
* a whole model with Q5_K and F16 matrices in several layers against the
  reference forward() given the same matrices dequantised to F32 (a format
  it computes): decode logits and a 64-token prefill within 1e-3."""
import os

import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, from_dev, rel_l2, to_dev
from tests.synth_model import gpu_blocks, synth_model

pytestmark = pytest.mark.gpu

Q5K, F16 = 13, 1


def _dev_blocks(gb, cuda, dt, rows, cols, seed, stream):
    nb = rows * (cols // gb.BLOCK_WIDTH[dt])
    buf = cuda.zeros(nb * gb.BLOCK_BYTES[dt] + 16, dtype=cuda.uint8, device="cuda")
    gb.synth_blocks(dt, buf, nb, seed, stream)
    cuda.cuda.synchronize()
    return buf, nb


@pytest.mark.parametrize("dt", [Q5K, F16])
def test_synth_and_dequant_bit_exact(gb, oracle, cuda, dt):
    rows, cols = 24, 512
    buf, nb = _dev_blocks(gb, cuda, dt, rows, cols, 7, 3)
    host = oracle.synth_blocks(dt, rows, cols, 7, 3)
    assert np.array_equal(from_dev(buf)[: host.size], host)
    out = cuda.empty(nb * gb.BLOCK_WIDTH[dt], dtype=cuda.float32, device="cuda")
    gb.dequant(dt, buf, nb, out)
    cuda.cuda.synchronize()
    assert np.array_equal(from_dev(out).view(np.uint32), oracle.dequant(dt, host).view(np.uint32))


@pytest.mark.parametrize("dt,rows,cols", [(Q5K, 16, 256), (Q5K, 100, 4096), (Q5K, 4096, 14336), (Q5K, 37, 2560),
                                          (F16, 16, 32), (F16, 300, 96), (F16, 4096, 4096), (F16, 77, 14336)])
def test_matvec_matches_fp64(gb, oracle, cuda, dt, rows, cols):
    buf, _ = _dev_blocks(gb, cuda, dt, rows, cols, 11, rows)
    x = oracle.synth_normal(cols, 11, 5)
    res = oracle.synth_normal(rows, 11, 6)
    y = cuda.full((rows,), float("nan"), dtype=cuda.float32, device="cuda")
    gb.matvec(dt, buf, rows, cols, to_dev(cuda, x), y, residual=to_dev(cuda, res))
    cuda.cuda.synchronize()
    assert gb.lib().gb_device_error(1) == 0
    Wf = oracle.dequant(dt, from_dev(buf)[: rows * (cols // gb.BLOCK_WIDTH[dt]) * gb.BLOCK_BYTES[dt]])
    ref = Wf.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64) + res
    got = from_dev(y)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-5, rel_l2(got, ref)


@pytest.mark.parametrize("dt,N,K,T", [(Q5K, 256, 1024, 130), (Q5K, 100, 512, 7), (F16, 200, 96, 40),
                                      (F16, 128, 2048, 256)])
def test_gemm_matches_fp64(gb, oracle, cuda, dt, N, K, T):
    buf, _ = _dev_blocks(gb, cuda, dt, N, K, 13, N + K)
    X = oracle.synth_normal(T * K, 13, T).reshape(T, K)
    Y = cuda.full((T, N), float("nan"), dtype=cuda.float32, device="cuda")
    gb.gemm(dt, buf, to_dev(cuda, X), Y, N, K, T)
    cuda.cuda.synchronize()
    assert gb.lib().gb_gemm_error(1) == 0
    Wf = oracle.dequant(dt, from_dev(buf)[: N * (K // gb.BLOCK_WIDTH[dt]) * gb.BLOCK_BYTES[dt]]).reshape(N, K)
    ref = X.astype(np.float64) @ Wf.astype(np.float64).T
    assert rel_l2(from_dev(Y), ref) <= 1e-5, rel_l2(from_dev(Y), ref)


def test_model_with_q5k_f16_matrices_matches_reference_f32(gb, oracle, cuda):
    """Layer 0 wq and layer 2 gate in Q5_K, layer 1 wv and ffn_down in F16 (the
    rest the Q4_K_M-style synthetic mix); the reference runs the same model
    with those four matrices dequantised to F32 by the oracle."""
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    SEED = 1234
    H, nh, nkv, L, ff, vocab, max_seq = 512, 8, 2, 4, 1536, 4096, 256
    oracle.ref().ref_set_threads(os.cpu_count() or 1)
    m = synth_model(oracle, H, nh, nkv, L, ff, vocab, max_seq, SEED, gen=gpu_blocks(gb, cuda))
    kv = nkv * (H // nh)
    shapes = [(H, H), (kv, H), (kv, H), (H, H), (ff, H), (ff, H), (H, ff)]
    swaps = [(0, 0, Q5K), (2, 4, Q5K), (1, 2, F16), (1, 6, F16)]
    dm = gb.DecodeModel(H, nh, nkv, L, ff, vocab, max_seq)
    keep = []
    try:
        dm.synthesize(SEED)
        for li, wi, dt in swaps:
            r, c = shapes[wi]
            buf, _ = _dev_blocks(gb, cuda, dt, r, c, SEED, 900 + 7 * li + wi)
            keep.append(buf)
            dm.set_matrix(li, wi, dt, buf)
            host = from_dev(buf)[: r * (c // gb.BLOCK_WIDTH[dt]) * gb.BLOCK_BYTES[dt]]
            m.layers[li].w[wi] = oracle.dequant(dt, host)   # fp32 rows for the reference
            m.layers[li].dtypes[wi] = 0
        ref = oracle.RefModel(m)
        try:
            prompt = np.random.RandomState(SEED).randint(0, vocab, 64).astype(np.int32)
            lr = ref.forward_tokens(prompt, 0)
            lg = np.zeros(vocab, np.float32)
            dm.prefill_host(prompt, 0, lg)
            assert rel_l2(lg, lr) <= REL_L2_TOL, rel_l2(lg, lr)
            token = oracle.argmax(lr)
            for pos in range(len(prompt), len(prompt) + 4):
                lr = ref.forward(int(token), pos)
                lg = np.zeros(vocab, np.float32)
                dm.decode_host(int(token), pos, lg)
                assert rel_l2(lg, lr) <= REL_L2_TOL, (pos, rel_l2(lg, lr))
                token = oracle.argmax(lr)
            assert dm.error() == 0
        finally:
            ref.close()
    finally:
        dm.close()
        oracle.ref().ref_set_threads(1)
