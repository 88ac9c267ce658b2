"""Q5_K and F16 weights in the oracle (formats the reference loader sizes but
rejects, src/engine/loader.c:98,117,586-651, so there is no reference kernel
to compile against).  The C restatement of GGML's published Q5_K layout
(block_q5_K: d, dmin, scales[12], qh[32], qs[128]) is checked against a second,
independent numpy restatement; F16 against numpy's IEEE half conversion (the
reference's extract_f16_to_f32, engine.c:183-212, is pinned to the same
mapping in test_oracle.py); the synthetic generators against their
definitions; the oracle matvec against an fp64 product of the dequantised rows."""
import numpy as np
import pytest


def _q5k_numpy(blocks: np.ndarray) -> np.ndarray:
    b = blocks.reshape(-1, 176)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    s = b[:, 4:16].astype(np.uint32)
    qh = b[:, 16:48].astype(np.uint32)
    qs = b[:, 48:176].astype(np.uint32)
    out = np.empty((b.shape[0], 256), np.float32)
    for j in range(8):
        if j < 4:
            sc, mn = s[:, j] & 63, s[:, j + 4] & 63
        else:
            sc = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            mn = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        nib = (qs[:, 32 * (j // 2):32 * (j // 2) + 32] >> (4 * (j % 2))) & 0xF
        q = nib + 16 * ((qh >> j) & 1)
        d1 = (d * sc.astype(np.float32)).astype(np.float32)
        m1 = (dmin * mn.astype(np.float32)).astype(np.float32)
        out[:, 32 * j:32 * j + 32] = (d1[:, None] * q.astype(np.float32)).astype(np.float32) - m1[:, None]
    return out.reshape(-1)


def test_q5k_dequant_matches_independent_restatement(oracle):
    W = oracle.synth_blocks(oracle.DT_Q5_K, 8, 1024, 3, 7)
    got = oracle.dequant(oracle.DT_Q5_K, W)
    assert np.array_equal(got.view(np.uint32), _q5k_numpy(W).view(np.uint32))
    # every fifth bit and both nibbles of the synthetic blocks are exercised
    assert set(np.unique(W.reshape(-1, 176)[:, 16:48])) > {0, 255}


def test_q5k_synth_shares_the_q4k_header_and_nibbles(oracle):
    q4 = oracle.synth_blocks(oracle.DT_Q4_K, 4, 512, 5, 9).reshape(-1, 144)
    q5 = oracle.synth_blocks(oracle.DT_Q5_K, 4, 512, 5, 9).reshape(-1, 176)
    assert np.array_equal(q5[:, :16], q4[:, :16])
    assert np.array_equal(q5[:, 48:], q4[:, 16:])


def test_f16_dequant_is_ieee(oracle):
    W = oracle.synth_blocks(oracle.DT_F16, 16, 256, 3, 2)
    got = oracle.dequant(oracle.DT_F16, W)
    assert np.array_equal(got, W.view(np.float16).astype(np.float32))
    # the generator: Irwin-Hall N(0,1) of synth_normal, times 2^-5, to half
    ref = (oracle.synth_normal(16 * 256, 3, 2) / 32).astype(np.float16)
    assert np.array_equal(W.view(np.float16), ref)


@pytest.mark.parametrize("dt,cols", [(13, 512), (13, 256), (1, 96), (1, 1024)])
def test_matvec_q5k_f16_against_fp64(oracle, dt, cols):
    rows = 37
    W = oracle.synth_blocks(dt, rows, cols, 4, 1)
    x = oracle.synth_normal(cols, 4, 2)
    rc, y = oracle.matvec(dt, W, rows, cols, x)
    assert rc == 0
    ref = oracle.dequant(dt, W).reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
    assert np.max(np.abs(y - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))
    # the reference kernels' error codes: ragged columns, short byte size
    assert oracle.matvec(dt, W, rows, cols + 1, x)[0] == -2
    assert oracle.matvec(dt, W, rows, cols, x, byte_size=W.size - 1)[0] == -3
