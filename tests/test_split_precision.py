"""The prefill GEMM's fp16 operand split, emulated in numpy on the CPU (no GPU):
the device code (guanaco_b200/csrc/gb_tc.cuh: split_tf32, split_f16x2,
f16_scale_exp) scales a row by a power of two so that max |x| < 2^15, keeps
the top 11 significant bits as hi (an add of half a unit and a mask on the
fp32 bits) and rounds the remainder to fp16 as lo; the tensor cores then sum
hi.hi + hi.lo + lo.hi.  Checked here: hi is exact in fp16, x = hi + lo to
about 2^-22 relative (plus an absolute floor from fp16 subnormals, 2^-25 at
the 2^15 scale), and a three-product dot product stays within a few 1e-7 of
fp64 for operands spread over forty binades."""
import numpy as np


def split_hi(x32):
    b = x32.view(np.uint32).astype(np.uint64)
    return ((b + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)


def scale_exp(m):
    E = (np.asarray(m, np.float32).view(np.uint32) >> 23) & 0xFF
    return np.where(E == 255, 0, np.where(E == 0, 126, np.clip(141 - E.astype(np.int64), -126, 126)))


def split_f16(x32):
    hi = split_hi(x32)
    lo = (x32 - hi).astype(np.float32)
    return hi.astype(np.float16), lo.astype(np.float16), hi


def test_scale_exponent_bounds():
    for m in [1e-30, 1e-5, 0.5, 1.0, 3.0, 1e3, 65504.0, 3e38]:
        e = int(scale_exp(m))
        s = float(m) * 2.0 ** e
        assert 2 ** 14 <= s < 2 ** 15, (m, e, s)
    assert int(scale_exp(0.0)) == 126 and int(scale_exp(np.inf)) == 0


def test_hi_exact_in_fp16_and_split_error():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(200000) * np.exp2(rng.uniform(-30, 10, 200000))).astype(np.float32)
    e = int(scale_exp(np.abs(x).max()))
    xs = (x * np.float32(2.0 ** e)).astype(np.float32)
    assert np.abs(xs).max() < 2 ** 15
    h16, l16, hi32 = split_f16(xs)
    normal = np.abs(hi32) >= 2.0 ** -14
    assert np.array_equal(h16[normal].astype(np.float32), hi32[normal])
    err = np.abs(xs.astype(np.float64) - h16.astype(np.float64) - l16.astype(np.float64))
    assert np.all(err <= 2.0 ** -22 * np.abs(xs) + 2.0 ** -24)


def test_three_product_dot_matches_fp64():
    rng = np.random.default_rng(5)
    K = 4096
    for _ in range(20):
        w = (rng.standard_normal(K) * np.exp2(rng.uniform(-20, 0, K))).astype(np.float32)
        x = (rng.standard_normal(K) * np.exp2(rng.uniform(-20, 20, K))).astype(np.float32)
        ew, ex = int(scale_exp(np.abs(w).max())), int(scale_exp(np.abs(x).max()))
        wh, wl, _ = split_f16((w * np.float32(2.0 ** ew)).astype(np.float32))
        xh, xl, _ = split_f16((x * np.float32(2.0 ** ex)).astype(np.float32))
        f = lambda a, b: a.astype(np.float64) * b.astype(np.float64)  # noqa: E731
        got = (f(wh, xh) + f(wh, xl) + f(wl, xh)).sum() * 2.0 ** (-ew - ex)
        ref = (w.astype(np.float64) * x.astype(np.float64)).sum()
        scale = (np.abs(w.astype(np.float64)) * np.abs(x.astype(np.float64))).sum()
        assert abs(got - ref) <= 1e-6 * scale, (got, ref, scale)
