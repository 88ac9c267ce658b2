"""CPU: pin the oracle restatement against the reference's known answers and
against the reference's own kernels (bit-exact)."""
import numpy as np
import pytest

from tests.helpers import rel_l2


def test_kat_q8_0(oracle, golden):
    # tests/test_quant.c:26-68 -- expected -528
    rc, y = oracle.matvec(oracle.DT_Q8_0, golden["kat_q8_0_blocks"], 1, 64, golden["kat_q8_0_x"])
    assert rc == 0 and y[0] == golden["kat_q8_0_expected"][0] == -528.0


def test_kat_q4k_uniform(oracle, golden):
    # tests/test_quant.c:94-139 -- expected 384
    rc, y = oracle.matvec(oracle.DT_Q4_K, golden["kat_q4k_uniform_blocks"], 1, 256, golden["kat_q4k_uniform_x"])
    assert rc == 0 and y[0] == 384.0


def test_kat_q4k_cross_byte_mapping(oracle, golden):
    # tests/test_quant.c:159-218 -- 6-bit scale/min cross-byte packing
    rc, y = oracle.matvec(oracle.DT_Q4_K, golden["kat_q4k_mapping_blocks"], 1, 256, golden["kat_q4k_mapping_x"])
    assert rc == 0 and abs(y[0] - golden["kat_q4k_mapping_expected"][0]) <= 1e-4


@pytest.mark.parametrize("dt,cols,err", [(4, 256, -3), (2, 64, -3)])
def test_byte_size_bound(oracle, dt, cols, err):
    # tests/test_quant.c:70-92, 220-242 -- byte_size one too small -> failure
    nb = 1 if dt == 4 else 2
    W = np.zeros(nb * oracle.block_bytes(dt), dtype=np.uint8)
    rc, _ = oracle.matvec(dt, W, 1, cols, np.zeros(cols, np.float32), byte_size=W.nbytes - 1)
    assert rc == err


@pytest.mark.parametrize("dt,cols", [(4, 300), (5, 100), (2, 33)])
def test_cols_not_block_multiple(oracle, dt, cols):
    W = np.zeros(4096, dtype=np.uint8)
    rc, _ = oracle.matvec(dt, W, 1, cols, np.zeros(cols + 64, np.float32))
    assert rc == -2


def _mv_keys(golden):
    return sorted({k.rsplit("_", 1)[0] for k in golden.files if k.startswith("mv_")})


def test_golden_matvec_bit_exact(oracle, golden):
    keys = _mv_keys(golden)
    assert len(keys) >= 12
    for key in keys:
        _, dt, shape = key.split("_")
        rows, cols = map(int, shape.split("x"))
        W, x, y_ref = golden[key + "_W"], golden[key + "_x"], golden[key + "_y"]
        # the seeded generators reproduce the fixture inputs byte for byte
        rc, y = oracle.matvec(int(dt), W, rows, cols, x)
        assert rc == 0
        assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32)), key


def test_golden_generators(oracle, golden):
    from tests.golden.make_golden import SEED, SHAPES
    for dt, shapes in SHAPES.items():
        for si, (rows, cols) in enumerate(shapes):
            key = f"mv_{dt}_{rows}x{cols}"
            assert np.array_equal(oracle.synth_blocks(dt, rows, cols, SEED, 100 + si), golden[key + "_W"]), key
            assert np.array_equal(oracle.synth_normal(cols, SEED, 200 + si), golden[key + "_x"]), key


def test_golden_dequant_bit_exact(oracle, golden):
    for dt in (oracle.DT_Q4_K, oracle.DT_Q8_0):
        out = oracle.dequant(dt, golden[f"dq_{dt}_blocks"])
        assert np.array_equal(out.view(np.uint32), golden[f"dq_{dt}_out"].view(np.uint32))


def test_golden_attention(oracle, golden):
    for name in ("attn_a", "attn_b", "attn_c"):
        nh, nkv, hd, ms, pos = map(int, golden[name + "_dims"])
        from tests.golden.make_golden import SEED
        q = oracle.synth_normal(nh * hd, SEED, 400)
        k = oracle.synth_normal(nkv * hd, SEED, 401)
        v = oracle.synth_normal(nkv * hd, SEED, 402)
        kc = oracle.synth_normal(nkv * ms * hd, SEED, 403)
        vc = oracle.synth_normal(nkv * ms * hd, SEED, 404)
        o, kc2, vc2 = oracle.attention_step(q, k, v, kc, vc, nh, nkv, hd, ms, pos)
        assert np.array_equal(o.view(np.uint32), golden[name + "_out"].view(np.uint32)), name
        assert np.array_equal(kc2.reshape(nkv, ms, hd)[:, pos], golden[name + "_krow"]), name
        assert np.array_equal(vc2.reshape(nkv, ms, hd)[:, pos], golden[name + "_vrow"]), name


def test_q6k_dequant_matches_matvec(oracle):
    # The Q6_K dequantiser is defined by the matvec's weight value: a one-hot x
    # picks one dequantised weight out of the matvec.
    W = oracle.synth_blocks(oracle.DT_Q6_K, 1, 256, 7, 7)
    deq = oracle.dequant(oracle.DT_Q6_K, W)
    for c in (0, 17, 31, 32, 63, 64, 100, 127, 128, 200, 255):
        x = np.zeros(256, np.float32)
        x[c] = 1.0
        rc, y = oracle.matvec(oracle.DT_Q6_K, W, 1, 256, x)
        assert rc == 0 and y[0] == deq[c]


def test_synth_distributions(oracle):
    z = oracle.synth_normal(1 << 18, 1, 2)
    assert abs(z.mean()) < 0.01 and abs(z.var() - 1.0) < 0.01
    W = oracle.synth_blocks(oracle.DT_Q4_K, 16, 4096, 1, 3).reshape(-1, 144)
    d = W[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert d.min() >= 0.99e-4 and d.max() <= 1.001e-3
    W6 = oracle.synth_blocks(oracle.DT_Q6_K, 16, 4096, 1, 4).reshape(-1, 210)
    sc = W6[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31


def test_f16_roundtrip(oracle):
    L = oracle.lib()
    for h in (0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x7C00, 0xFC00, 0x068D):
        f = L.gbo_f16_to_f32(h)
        assert np.float16(f).view(np.uint16) == h or np.isnan(f)
        assert L.gbo_f32_to_f16(f) == h
    rng = np.random.default_rng(0)
    for f in rng.uniform(-70000, 70000, 2000).astype(np.float32).tolist() + \
            rng.uniform(-1e-4, 1e-4, 2000).astype(np.float32).tolist():
        assert L.gbo_f32_to_f16(f) == np.float32(f).astype(np.float16).view(np.uint16), f


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()")
@pytest.mark.parametrize("threads", [1, 4])
def test_live_against_reference(oracle, threads):
    oracle.ref().ref_set_threads(threads)
    try:
        for dt, rows, cols, seed in [(4, 96, 4096, 5), (5, 40, 14336, 6), (2, 50, 4096, 7), (5, 3, 5632, 8)]:
            W = oracle.synth_blocks(dt, rows, cols, seed, 1)
            x = oracle.synth_normal(cols, seed, 2)
            _, y = oracle.matvec(dt, W, rows, cols, x)
            _, yr = oracle.ref_matvec(dt, W, rows, cols, x)
            assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
            assert rel_l2(y, yr) == 0.0
    finally:
        oracle.ref().ref_set_threads(1)
