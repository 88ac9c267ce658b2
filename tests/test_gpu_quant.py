"""GPU parity: Q4_K / Q6_K / Q8_0 dequantisation (bit-exact) and fused
dequant+matvec (relative L2 <= 1e-3 against the oracle, which is bit-exact
with the reference CPU kernels)."""
import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, device_x, from_dev, rel_l2, to_dev

pytestmark = pytest.mark.gpu

DTS = {"q4k": 4, "q6k": 5, "q8_0": 2}


def dev_blocks(cuda, host_bytes, pad=16):
    t = cuda.zeros(host_bytes.size + pad, dtype=cuda.uint8, device="cuda")
    t[: host_bytes.size] = to_dev(cuda, host_bytes)
    return t


@pytest.mark.parametrize("name", list(DTS))
def test_synth_bytes_match_cpu_generator(gb, oracle, cuda, name):
    dt = DTS[name]
    rows, cols = 37, 512 if dt != 2 else 224
    host = oracle.synth_blocks(dt, rows, cols, 1234, 9)
    nblk = host.size // oracle.block_bytes(dt)
    d = cuda.zeros(host.size + 16, dtype=cuda.uint8, device="cuda")
    gb.synth_blocks(dt, d, nblk, 1234, 9)
    cuda.cuda.synchronize()
    assert np.array_equal(from_dev(d)[: host.size], host)
    x = cuda.empty(1001, dtype=cuda.float32, device="cuda")
    gb.synth_normal(x, 1001, 77, 5)
    cuda.cuda.synchronize()
    assert np.array_equal(from_dev(x), oracle.synth_normal(1001, 77, 5))


def special_blocks(oracle, dt, n):
    """Seeded blocks whose fp16 scales are overwritten with edge values:
    subnormals, zero, negative, large, Inf and NaN."""
    B = oracle.synth_blocks(dt, n, 256 if dt != 2 else 32, 3, 3).reshape(n, -1).copy()
    specials = np.array([0x0001, 0x03FF, 0x0000, 0x8000, 0xBC00, 0x7BFF, 0x7C00, 0xFE01, 0x0400, 0x3555],
                        dtype=np.uint16)
    off = {4: [0, 2], 5: [208], 2: [0]}[dt]
    for i in range(n):
        for o in off:
            B[i, o:o + 2] = np.frombuffer(specials[(i + o) % specials.size].tobytes(), np.uint8)
    return B.ravel()


@pytest.mark.parametrize("name", list(DTS))
def test_dequant_bit_exact(gb, oracle, cuda, name):
    dt = DTS[name]
    for host in (oracle.synth_blocks(dt, 64, 1024, 11, 1), special_blocks(oracle, dt, 20)):
        nblk = host.size // oracle.block_bytes(dt)
        d = dev_blocks(cuda, host)
        out = cuda.empty(nblk * (256 if dt != 2 else 32), dtype=cuda.float32, device="cuda")
        gb.dequant(dt, d, nblk, out)
        cuda.cuda.synchronize()
        got = from_dev(out)
        want = oracle.dequant(dt, host)
        # bit-exact wherever the result is a number; NaN wherever the
        # reference produces NaN (the NaN bit pattern an invalid operation
        # creates is platform-defined: 0xFFC00000 on x86, 0x7FFFFFFF here)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_dequant_matches_golden(gb, cuda, golden):
    for dt in (4, 2):
        host = golden[f"dq_{dt}_blocks"]
        nblk = host.size // (144 if dt == 4 else 34)
        out = cuda.empty(nblk * (256 if dt == 4 else 32), dtype=cuda.float32, device="cuda")
        gb.dequant(dt, dev_blocks(cuda, host), nblk, out)
        cuda.cuda.synchronize()
        assert np.array_equal(from_dev(out).view(np.uint32), golden[f"dq_{dt}_out"].view(np.uint32))


def run_matvec(gb, cuda, dt, W_host, rows, cols, x_host, residual=None):
    W = dev_blocks(cuda, W_host)
    x = to_dev(cuda, x_host)
    y = cuda.full((rows,), float("nan"), dtype=cuda.float32, device="cuda")
    r = to_dev(cuda, residual) if residual is not None else None
    gb.matvec(dt, W, rows, cols, x, y, residual=r)
    cuda.cuda.synchronize()
    return from_dev(y)


SHAPES = [(1, 256), (3, 512), (5, 768), (17, 1024), (33, 2048), (100, 4096), (129, 1280), (7, 5632), (64, 14336)]


@pytest.mark.parametrize("name", list(DTS))
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_parity(gb, oracle, cuda, name, rows, cols):
    dt = DTS[name]
    W = oracle.synth_blocks(dt, rows, cols, 1234, rows * 7 + cols)
    x = oracle.synth_normal(cols, 1234, cols)
    rc, y_ref = oracle.matvec(dt, W, rows, cols, x)
    assert rc == 0
    y = run_matvec(gb, cuda, dt, W, rows, cols, x)
    assert np.all(np.isfinite(y))
    assert rel_l2(y, y_ref) <= REL_L2_TOL
    # far inside the tolerance: Q8_0 accumulates in fp32; Q4_K / Q6_K carry x
    # as three int8 limbs per sub-block (fp32's 24 bits) into the tensor cores
    assert rel_l2(y, y_ref) <= 1e-5
    assert gb.lib().gb_device_error(1) == 0


@pytest.mark.parametrize("name", list(DTS))
@pytest.mark.parametrize("rows,cols", [(100, 4096), (64, 14336), (4096, 4096)])
@pytest.mark.parametrize("pattern", ["every_subblock", "one_subblock", "channel_1e3_and_tiny"])
def test_matvec_outlier_activations(gb, oracle, cuda, name, rows, cols, pattern):
    """Hidden states of real models carry outlier channels 100-1000x the
    median.  The Q4_K / Q6_K matvecs carry x as three int8 limbs scaled per
    32-column sub-block, so an outlier sets the scale of its 31 neighbours;
    with 24 bits they keep fp32-like precision (well inside the 1e-3
    relative-L2 bound)."""
    dt = DTS[name]
    W = oracle.synth_blocks(dt, rows, cols, 99, rows + cols)
    x = oracle.synth_normal(cols, 99, 3).copy()
    if pattern == "every_subblock":        # one channel at 1e3 in every 32-column sub-block
        x[7::32] = 1e3
    elif pattern == "one_subblock":        # a single outlier channel
        x[cols // 2 + 5] = -1e3
    else:                                  # outliers beside values of 1e-4 x the median
        x[::32] = 1e3
        x[1::32] *= 1e-4
    rc, y_ref = oracle.matvec(dt, W, rows, cols, x)
    assert rc == 0
    y = run_matvec(gb, cuda, dt, W, rows, cols, x)
    assert np.all(np.isfinite(y))
    err = rel_l2(y, y_ref)
    assert err <= REL_L2_TOL, err
    assert err <= 1e-5, err
    assert gb.lib().gb_device_error(1) == 0


@pytest.mark.parametrize("name", ["q4k", "q6k"])
@pytest.mark.parametrize("rows,cols", [(100, 4096), (64, 14336), (1024, 4096), (77, 2048), (40, 5632)])
@pytest.mark.parametrize("xkind", ["normal", "positive", "outlier"])
def test_matvec_is_exact_on_the_device_x(gb, oracle, cuda, name, rows, cols, xkind):
    """The only approximation of the Q4_K / Q6_K matvecs is x carried as three
    int8 limbs per sub-block (24 significant bits, as fp32): given that x~,
    the result is W . x~ up to fp32 rounding, and it is as close to the
    reference's fp32 result as fp32 arithmetic in another summation order
    is.  A consumer that mixed x and x~ (e.g. the Q6_K -32 code offset
    applied with the sum of the exact x) shows up here as an error
    correlated across rows, which a decoder stack amplifies."""
    dt = DTS[name]
    W = oracle.synth_blocks(dt, rows, cols, 7, rows * 3 + cols)
    x = oracle.synth_normal(cols, 7, 11)
    if xkind == "positive":   # a common-mode component, as hidden states of the synthetic models have
        x = (np.abs(x) + 0.5).astype(np.float32)
    elif xkind == "outlier":
        x[5::32] *= 1e3
    # the ring kernel (Q6_K rows that are not a multiple of 8 blocks) scales x per 16 columns
    group = 16 if dt == 5 and (cols // 256) % 8 else 32
    _, y_exact = oracle.matvec(dt, W, rows, cols, x)
    _, y_q = oracle.matvec(dt, W, rows, cols, device_x(x, group))
    y = run_matvec(gb, cuda, dt, W, rows, cols, x)
    grow = max(1.0, np.sqrt(cols / 4096))   # fp32 rounding of the sums grows with sqrt(K)
    assert rel_l2(y, y_q) <= 2e-6 * grow, rel_l2(y, y_q)
    assert rel_l2(y, y_exact) <= 3e-6 * grow, rel_l2(y, y_exact)
    # the errors summed over the rows are no larger than fp32 rounding gives
    e = y.astype(np.float64) - y_exact
    assert abs(e.sum()) <= 4.0 * np.sqrt(np.sum(e * e)) * max(1.0, np.sqrt(rows) / 8) + 1e-7 * np.abs(y_exact).sum()


@pytest.mark.parametrize("rows,cols", [(3, 32), (9, 96), (31, 160), (300, 4128)])
def test_matvec_q8_0_ragged_columns(gb, oracle, cuda, rows, cols):
    W = oracle.synth_blocks(2, rows, cols, 5, cols)
    x = oracle.synth_normal(cols, 5, 1)
    _, y_ref = oracle.matvec(2, W, rows, cols, x)
    assert rel_l2(run_matvec(gb, cuda, 2, W, rows, cols, x), y_ref) <= 1e-5


def test_matvec_golden_vectors(gb, cuda, golden):
    keys = sorted({k.rsplit("_", 1)[0] for k in golden.files if k.startswith("mv_")})
    for key in keys:
        _, dt, shape = key.split("_")
        rows, cols = map(int, shape.split("x"))
        y = run_matvec(gb, cuda, int(dt), golden[key + "_W"], rows, cols, golden[key + "_x"])
        assert rel_l2(y, golden[key + "_y"]) <= REL_L2_TOL, key


def test_matvec_residual_epilogue(gb, oracle, cuda):
    rows, cols = 513, 2048
    W = oracle.synth_blocks(4, rows, cols, 2, 2)
    x = oracle.synth_normal(cols, 2, 3)
    r = oracle.synth_normal(rows, 2, 4)
    _, y_ref = oracle.matvec(4, W, rows, cols, x)
    y = run_matvec(gb, cuda, 4, W, rows, cols, x, residual=r)
    assert rel_l2(y, y_ref + r) <= 1e-4


@pytest.mark.parametrize("name", list(DTS))
def test_matvec_kat_values(gb, cuda, golden, name):
    dt = DTS[name]
    if dt == 2:
        y = run_matvec(gb, cuda, 2, golden["kat_q8_0_blocks"], 1, 64, golden["kat_q8_0_x"])
        assert abs(y[0] - (-528.0)) <= 1e-4
    elif dt == 4:
        y = run_matvec(gb, cuda, 4, golden["kat_q4k_uniform_blocks"], 1, 256, golden["kat_q4k_uniform_x"])
        assert abs(y[0] - 384.0) <= 1e-4
        y = run_matvec(gb, cuda, 4, golden["kat_q4k_mapping_blocks"], 1, 256, golden["kat_q4k_mapping_x"])
        assert abs(y[0] - golden["kat_q4k_mapping_expected"][0]) <= 1e-4
    else:
        # Q6_K has no reference KAT; use an all-scales-one block: w = d*(q-32)
        B = np.zeros(210, np.uint8)
        B[192:208] = 1
        B[208:210] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)   # d = 1
        B[0:128] = 0x21   # low nibbles 1, high nibbles 2; qh = 0 -> q in {1, 2}
        y = run_matvec(gb, cuda, 5, B, 1, 256, np.ones(256, np.float32))
        assert y[0] == 128 * (1 - 32) + 128 * (2 - 32)


def test_matvec_error_codes(gb, cuda):
    L = gb.lib()
    W = cuda.zeros(4096, dtype=cuda.uint8, device="cuda")
    x = cuda.zeros(1024, dtype=cuda.float32, device="cuda")
    y = cuda.zeros(16, dtype=cuda.float32, device="cuda")
    s = cuda.cuda.current_stream().cuda_stream
    assert L.gb_matvec(4, W.data_ptr(), 1, 300, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_ESHAPE
    assert L.gb_matvec(2, W.data_ptr(), 1, 33, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_ESHAPE
    assert L.gb_matvec(4, None, 1, 256, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_EINVAL
    assert L.gb_matvec(7, W.data_ptr(), 1, 256, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_EINVAL
    assert L.gb_matvec(4, W.data_ptr() + 8, 1, 256, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_EINVAL
    assert L.gb_matvec(5, W.data_ptr() + 2, 1, 256, x.data_ptr(), y.data_ptr(), None, s) == gb.GB_EINVAL
    assert L.gb_matvec(4, W.data_ptr(), 1, 256, x.data_ptr() + 4, y.data_ptr(), None, s) == gb.GB_EINVAL


@pytest.mark.parametrize("dt,rows,cols", [(4, 4096, 4096), (5, 4096, 14336), (5, 128256, 4096), (4, 14336, 4096)])
def test_matvec_benchmark_shapes(gb, oracle, cuda, dt, rows, cols):
    """The BASELINE configs at full size, checked against the oracle on every row."""
    W = oracle.synth_blocks(dt, rows, cols, 1234, 1)
    x = oracle.synth_normal(cols, 1234, 2)
    _, y_ref = oracle.matvec(dt, W, rows, cols, x)
    y = run_matvec(gb, cuda, dt, W, rows, cols, x)
    assert rel_l2(y, y_ref) <= REL_L2_TOL
    assert np.max(np.abs(y - y_ref)) <= 1e-4 * max(1.0, np.max(np.abs(y_ref)))


def test_vtable_slots(gb, oracle, cuda, golden):
    """backend_cuda_create's quantised slots, called like the engine does,
    for device-resident and host-only (lazily uploaded) tensors."""
    be = gb.CudaBackend()
    try:
        for dt, rows, cols in [(4, 64, 1024), (5, 48, 2048), (2, 33, 512)]:
            W = oracle.synth_blocks(dt, rows, cols, 3, dt)
            x = oracle.synth_normal(cols, 3, 9)
            _, y_ref = oracle.matvec(dt, W, rows, cols, x)
            # host-only tensor: uploaded on first use
            t = gb.make_tensor(dt, W, rows, cols)
            y = np.zeros(rows, np.float32)
            assert be.matvec(t, x, y) == 0
            assert rel_l2(y, y_ref) <= REL_L2_TOL
            # resident tensor through cuda_upload_weight (the loader's path)
            d = gb.lib().cuda_upload_weight(W.ctypes.data, W.nbytes)
            assert d
            t2 = gb.make_tensor(dt, W, rows, cols, d_data=d)
            y2 = np.zeros(rows, np.float32)
            assert be.matvec(t2, x, y2) == 0
            assert rel_l2(y2, y_ref) <= REL_L2_TOL
            # reference error convention
            t3 = gb.make_tensor(dt, W, rows, cols, byte_size=W.nbytes - 1)
            assert be.matvec(t3, x, y2) == -3
        t4 = gb.make_tensor(4, golden["kat_q4k_uniform_blocks"], 1, 256)
        t4.dtype = 5   # wrong dtype for the Q4_K slot
        assert be.kernels.matvec_q4k_f32(gb.C.byref(t4), golden["kat_q4k_uniform_x"].ctypes.data,
                                         np.zeros(1, np.float32).ctypes.data) == -1
        t5 = gb.make_tensor(4, golden["kat_q4k_uniform_blocks"], 1, 256)
        out = np.zeros(1, np.float32)
        assert be.matvec(t5, golden["kat_q4k_uniform_x"], out) == 0 and out[0] == 384.0
    finally:
        be.close()


def test_cuda_matvec_q4k_impl_parity(gb, oracle):
    """tests/test_quant.c:249-303: 32x1024 Q4_K, CPU vs GPU, abs tol 1e-4."""
    rows, cols = 32, 1024
    B = np.zeros((rows * 4, 144), np.uint8)
    B[:, 0:2] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    B[:, 2:4] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    B[:, 4:16] = np.arange(12, dtype=np.uint8) % 8
    B[:, 16:144] = np.arange(128, dtype=np.uint8)
    B = B.ravel()
    x = (np.arange(cols, dtype=np.float32) / 1024.0).astype(np.float32)
    _, y_cpu = oracle.matvec(4, B, rows, cols, x)
    d = gb.lib().cuda_upload_weight(B.ctypes.data, B.nbytes)
    y = np.zeros(rows, np.float32)
    assert gb.lib().cuda_matvec_q4k_f32_impl(d, x.ctypes.data, y.ctypes.data, rows, cols) == 0
    assert np.max(np.abs(y - y_cpu)) <= 1e-4 * max(1.0, np.abs(y_cpu).max())


@pytest.mark.parametrize("dt,rows,cols", [(4, 1000, 16384), (5, 1000, 16384), (4, 4099, 4096), (5, 77, 2048)])
def test_matvec_split_groups_deterministic(gb, oracle, cuda, dt, rows, cols):
    """Groups split across CTAs finish through the ticketed partials: two calls
    in a row agree bit for bit (fixed summation order) and with the oracle."""
    W = oracle.synth_blocks(dt, rows, cols, 99, rows + cols)
    x = oracle.synth_normal(cols, 99, 1)
    _, y_ref = oracle.matvec(dt, W, rows, cols, x)
    y1 = run_matvec(gb, cuda, dt, W, rows, cols, x)
    y2 = run_matvec(gb, cuda, dt, W, rows, cols, x)
    assert np.array_equal(y1, y2)
    assert rel_l2(y1, y_ref) <= 1e-4
    assert gb.lib().gb_device_error(1) == 0


@pytest.mark.parametrize("dt,rows,cols", [(4, 4096, 4096), (5, 4096, 14336), (4, 50, 256)])
def test_matvec_in_place_residual(gb, oracle, cuda, dt, rows, cols):
    """y = residual + W x with y and residual the same buffer (the decode
    layer's hidden += W x)."""
    W = oracle.synth_blocks(dt, rows, cols, 7, 8)
    x = oracle.synth_normal(cols, 7, 9)
    r = oracle.synth_normal(rows, 7, 10)
    _, y_ref = oracle.matvec(dt, W, rows, cols, x)
    dW = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    dW[: W.size] = cuda.from_numpy(W).cuda()
    dx = cuda.from_numpy(x).cuda()
    h = cuda.from_numpy(r.copy()).cuda()
    gb.matvec(dt, dW, rows, cols, dx, h, residual=h)
    cuda.cuda.synchronize()
    assert rel_l2(h.cpu().numpy(), y_ref + r) <= 1e-4


def test_matvec_two_streams(gb, oracle, cuda):
    """Calls on different streams use different workspaces."""
    rows, cols = 3000, 4096
    Ws = [oracle.synth_blocks(4, rows, cols, 3, s) for s in (1, 2)]
    x = oracle.synth_normal(cols, 3, 3)
    refs = [oracle.matvec(4, W, rows, cols, x)[1] for W in Ws]
    dWs = []
    for W in Ws:
        d = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
        d[: W.size] = cuda.from_numpy(W).cuda()
        dWs.append(d)
    dx = cuda.from_numpy(x).cuda()
    streams = [cuda.cuda.Stream() for _ in range(2)]
    ys = [cuda.empty(rows, dtype=cuda.float32, device="cuda") for _ in range(2)]
    cuda.cuda.synchronize()
    for it in range(20):
        for i in range(2):
            gb.matvec(4, dWs[i], rows, cols, dx, ys[i], stream=streams[i].cuda_stream)
    cuda.cuda.synchronize()
    for i in range(2):
        assert rel_l2(ys[i].cpu().numpy(), refs[i]) <= 1e-4


@pytest.mark.parametrize("dt,rows,cols", [(4, 14336, 4096), (5, 4096, 14336), (4, 33, 512)])
def test_matvec_captured_without_workspace(gb, oracle, cuda, dt, rows, cols):
    """First use on a stream that is being captured: no workspace can be made,
    so the launch splits by whole row groups; the graph replays correctly."""
    W = oracle.synth_blocks(dt, rows, cols, 11, 12)
    x = oracle.synth_normal(cols, 11, 13)
    _, y_ref = oracle.matvec(dt, W, rows, cols, x)
    dW = cuda.zeros(W.size + 16, dtype=cuda.uint8, device="cuda")
    dW[: W.size] = cuda.from_numpy(W).cuda()
    dx = cuda.from_numpy(x).cuda()
    y = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    cuda.cuda.synchronize()
    g = cuda.cuda.CUDAGraph()
    with cuda.cuda.graph(g, capture_error_mode="relaxed"):
        gb.matvec(dt, dW, rows, cols, dx, y)
    g.replay()
    cuda.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), y_ref) <= 1e-4
    del g


def test_vtable_host_cache_detects_reuse(gb, oracle, cuda):
    """A host weight buffer rewritten at the same address (as a freed and
    reallocated numpy array can be) is uploaded again, not served stale."""
    be = gb.CudaBackend()
    try:
        rows, cols = 40, 2048
        W = oracle.synth_blocks(5, rows, cols, 21, 1)
        x = oracle.synth_normal(cols, 21, 2)
        t = gb.make_tensor(5, W, rows, cols)
        y = np.zeros(rows, np.float32)
        assert be.matvec(t, x, y) == 0
        assert rel_l2(y, oracle.matvec(5, W, rows, cols, x)[1]) <= 1e-4
        W[:] = oracle.synth_blocks(5, rows, cols, 21, 2)   # same address, new content
        assert be.matvec(t, x, y) == 0
        assert rel_l2(y, oracle.matvec(5, W, rows, cols, x)[1]) <= 1e-4
    finally:
        be.close()


def test_vtable_cache_clear_after_in_place_edit(gb, oracle, cuda, monkeypatch):
    """An edit in place that the sampled checksum cannot see (one block of one
    row) is picked up after gb_vtable_cache_clear; the cache also evicts
    least recently used copies above its byte cap."""
    be = gb.CudaBackend()
    try:
        rows, cols = 64, 4096
        W = oracle.synth_blocks(4, rows, cols, 31, 1)
        x = oracle.synth_normal(cols, 31, 2)
        t = gb.make_tensor(4, W, rows, cols)
        y = np.zeros(rows, np.float32)
        assert be.matvec(t, x, y) == 0
        blk = 144 * (cols // 256)
        W[7 * blk + 20: 7 * blk + 40] ^= 0x5A   # row 7, inside its first block's quants
        assert gb.lib().gb_vtable_cache_clear() == 0
        assert be.matvec(t, x, y) == 0
        assert rel_l2(y, oracle.matvec(4, W, rows, cols, x)[1]) <= 1e-5
        # many distinct tensors: every result stays right while older copies are evicted
        for i in range(6):
            Wi = oracle.synth_blocks(4, rows, cols, 31, 10 + i)
            ti = gb.make_tensor(4, Wi, rows, cols)
            assert be.matvec(ti, x, y) == 0
            assert rel_l2(y, oracle.matvec(4, Wi, rows, cols, x)[1]) <= 1e-5
    finally:
        be.close()
        gb.lib().gb_vtable_cache_clear()


@pytest.mark.parametrize("dts,rows,cols", [
    ((4, 4), (14336, 14336), 4096),        # gate / up
    ((4, 4, 5), (4096, 1024, 1024), 4096),   # q / k / v: Q6_K v, mixed formats in one launch
    ((4, 5), (96, 40), 2048),               # short, ragged rows
    ((4, 2), (64, 64), 512),                # Q8_0 is off the grouped path: one launch per matrix
])
def test_matvec_group_matches_single(gb, oracle, cuda, dts, rows, cols):
    """Matrices sharing x in one launch give each product within the
    matvec tolerance of the oracle and of its own single launch."""
    x_host = oracle.synth_normal(cols, 91, 1)
    Ws, refs = [], []
    for i, (dt, r) in enumerate(zip(dts, rows)):
        W = oracle.synth_blocks(dt, r, cols, 91, 10 + i)
        Ws.append(dev_blocks(cuda, W))
        refs.append(oracle.matvec(dt, W, r, cols, x_host)[1])
    x = to_dev(cuda, x_host)
    ys = [cuda.empty(r, dtype=cuda.float32, device="cuda") for r in rows]
    gb.matvec_group(list(dts), Ws, list(rows), cols, x, ys)
    singles = [cuda.empty(r, dtype=cuda.float32, device="cuda") for r in rows]
    for dt, W, r, y1 in zip(dts, Ws, rows, singles):
        gb.matvec(dt, W, r, cols, x, y1)
    cuda.cuda.synchronize()
    assert gb.lib().gb_device_error(1) == 0
    for y, y1, ref in zip(ys, singles, refs):
        assert rel_l2(from_dev(y), ref) <= 1e-4
        assert rel_l2(from_dev(y), from_dev(y1)) <= 1e-5


def test_matvec_chain_reads_predecessor_output(gb, oracle, cuda):
    """Public matvec calls launch with programmatic dependent launch, so a
    call starts fetching weights while the one before it on the stream is
    still running.  A chain whose every x (and residual) is the previous
    call's y, issued with no synchronisation in between and repeated with
    new inputs, must give each product of the values its predecessor wrote."""
    H, F = 4096, 14336
    mats = [(4, H, H, 1), (4, H, H, 2), (5, F, H, 3), (5, H, F, 4)]
    Wh = [oracle.synth_blocks(dt, r, c, 55, s) for dt, r, c, s in mats]
    Wd = [dev_blocks(cuda, w) for w in Wh]
    Gh = [oracle.synth_blocks(4, 1024, H, 55, 10 + i) for i in range(2)]
    Gd = [dev_blocks(cuda, w) for w in Gh]
    y = [cuda.empty(r, dtype=cuda.float32, device="cuda") for _, r, _, _ in mats]
    g = [cuda.empty(1024, dtype=cuda.float32, device="cuda") for _ in range(2)]
    for it in range(3):
        x_host = oracle.synth_normal(H, 56, it)
        x = to_dev(cuda, x_host)
        cuda.cuda.synchronize()
        gb.matvec(4, Wd[0], H, H, x, y[0])                        # y0 = W0 x
        gb.matvec(4, Wd[1], H, H, y[0], y[1], residual=y[0])      # y1 = W1 y0 + y0
        gb.matvec(5, Wd[2], F, H, y[1], y[2])                     # y2 = W2 y1
        gb.matvec(5, Wd[3], H, F, y[2], y[3], residual=y[1])      # y3 = W3 y2 + y1
        gb.matvec_group([4, 4], Gd, [1024, 1024], H, y[3], g)     # g = G y3
        cuda.cuda.synchronize()
        assert gb.lib().gb_device_error(1) == 0
        got = [from_dev(t) for t in y] + [from_dev(t) for t in g]
        # every product against the oracle applied to what the GPU wrote before it
        assert rel_l2(got[0], oracle.matvec(4, Wh[0], H, H, x_host)[1]) <= REL_L2_TOL
        assert rel_l2(got[1], oracle.matvec(4, Wh[1], H, H, got[0])[1] + got[0]) <= REL_L2_TOL
        assert rel_l2(got[2], oracle.matvec(5, Wh[2], F, H, got[1])[1]) <= REL_L2_TOL
        assert rel_l2(got[3], oracle.matvec(5, Wh[3], H, F, got[2])[1] + got[1]) <= REL_L2_TOL
        for i in range(2):
            assert rel_l2(got[4 + i], oracle.matvec(4, Gh[i], 1024, H, got[3])[1]) <= REL_L2_TOL, it
