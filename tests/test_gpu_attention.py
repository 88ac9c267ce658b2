"""GPU parity: RoPE + KV append + split-K GQA decode attention against the
oracle (engine.c:372-509 composition).  The appended K/V rows must be
bit-exact (RoPE is evaluated with the reference's float formula); the
attention output within relative L2 1e-3."""
import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, from_dev, rel_l2, to_dev

pytestmark = pytest.mark.gpu


def run_attention(gb, cuda, q, k, v, kc, vc, nh, nkv, hd, ms, pos, theta=500000.0):
    dq, dk, dv = to_dev(cuda, q), to_dev(cuda, k), to_dev(cuda, v)
    dkc, dvc = to_dev(cuda, kc), to_dev(cuda, vc)
    cs = cuda.empty(ms * hd, dtype=cuda.float32, device="cuda")
    gb.rope_table(cs, ms, hd, theta)
    ws = cuda.zeros(gb.attn_workspace_bytes(nh, nkv, hd, ms), dtype=cuda.uint8, device="cuda")
    d_pos = cuda.tensor([pos], dtype=cuda.int32, device="cuda")
    out = cuda.full((nh * hd,), float("nan"), dtype=cuda.float32, device="cuda")
    gb.attention_decode(dq, dk, dv, dkc, dvc, cs, d_pos, nh, nkv, hd, ms, out, ws)
    cuda.cuda.synchronize()
    return from_dev(out), from_dev(dkc), from_dev(dvc), ws


CASES = [
    # (n_heads, n_kv, head_dim, max_seq, pos)
    (8, 2, 128, 80, 0), (8, 2, 128, 80, 1), (8, 2, 128, 80, 31), (8, 2, 128, 80, 32), (8, 2, 128, 80, 79),
    (8, 8, 128, 64, 40), (16, 2, 128, 300, 257), (32, 4, 64, 300, 200), (8, 1, 64, 40, 0),
    (16, 2, 64, 130, 129), (4, 4, 64, 700, 650), (32, 8, 128, 2100, 2049),
    (8, 2, 64, 40, 9), (8, 2, 64, 40, 13), (16, 4, 64, 600, 333), (4, 2, 128, 100, 70),
    # one KV head of 4 q heads over a long context (a rank's share at 8-way tensor parallelism)
    (4, 1, 128, 4400, 4300),
]


@pytest.mark.parametrize("nh,nkv,hd,ms,pos", CASES)
def test_attention_parity(gb, oracle, cuda, nh, nkv, hd, ms, pos):
    seed = nh * 1000 + pos
    q = oracle.synth_normal(nh * hd, seed, 1)
    k = oracle.synth_normal(nkv * hd, seed, 2)
    v = oracle.synth_normal(nkv * hd, seed, 3)
    kc = oracle.synth_normal(nkv * ms * hd, seed, 4)
    vc = oracle.synth_normal(nkv * ms * hd, seed, 5)
    o_ref, kc_ref, vc_ref = oracle.attention_step(q, k, v, kc, vc, nh, nkv, hd, ms, pos)
    o, kc_g, vc_g, _ = run_attention(gb, cuda, q, k, v, kc, vc, nh, nkv, hd, ms, pos)
    assert rel_l2(o, o_ref) <= REL_L2_TOL
    assert rel_l2(o, o_ref) <= 1e-5
    # append is bit-exact and touches only slot pos
    assert np.array_equal(kc_g.view(np.uint32), kc_ref.view(np.uint32))
    assert np.array_equal(vc_g.view(np.uint32), vc_ref.view(np.uint32))


def test_attention_golden(gb, cuda, golden, oracle):
    from tests.golden.make_golden import SEED
    for name in ("attn_a", "attn_b", "attn_c"):
        nh, nkv, hd, ms, pos = map(int, golden[name + "_dims"])
        q = oracle.synth_normal(nh * hd, SEED, 400)
        k = oracle.synth_normal(nkv * hd, SEED, 401)
        v = oracle.synth_normal(nkv * hd, SEED, 402)
        kc = oracle.synth_normal(nkv * ms * hd, SEED, 403)
        vc = oracle.synth_normal(nkv * ms * hd, SEED, 404)
        o, kc_g, vc_g, _ = run_attention(gb, cuda, q, k, v, kc, vc, nh, nkv, hd, ms, pos)
        assert rel_l2(o, golden[name + "_out"]) <= REL_L2_TOL, name
        assert np.array_equal(kc_g.reshape(nkv, ms, hd)[:, pos], golden[name + "_krow"]), name
        assert np.array_equal(vc_g.reshape(nkv, ms, hd)[:, pos], golden[name + "_vrow"]), name


def test_attention_config2_full_size(gb, oracle, cuda):
    """32 q heads, 8 KV heads, hd 128, context filled to
    8192, append at 8192, attend over 8193 positions (max_seq 8448)."""
    nh, nkv, hd, ms, pos = 32, 8, 128, 8448, 8192
    q = oracle.synth_normal(nh * hd, 1234, 11)
    k = oracle.synth_normal(nkv * hd, 1234, 12)
    v = oracle.synth_normal(nkv * hd, 1234, 13)
    kc = oracle.synth_normal(nkv * ms * hd, 1234, 14)
    vc = oracle.synth_normal(nkv * ms * hd, 1234, 15)
    o_ref, kc_ref, vc_ref = oracle.attention_step(q, k, v, kc, vc, nh, nkv, hd, ms, pos)
    o, kc_g, vc_g, ws = run_attention(gb, cuda, q, k, v, kc, vc, nh, nkv, hd, ms, pos)
    assert rel_l2(o, o_ref) <= REL_L2_TOL
    assert np.array_equal(kc_g.reshape(nkv, ms, hd)[:, pos], kc_ref.reshape(nkv, ms, hd)[:, pos])
    assert np.array_equal(vc_g.reshape(nkv, ms, hd)[:, pos], vc_ref.reshape(nkv, ms, hd)[:, pos])
    # the split tickets are re-armed (all zero) after the launch
    nticket = nkv + 1
    tickets = from_dev(ws).view(np.uint32)[-nticket:]
    assert np.all(tickets == 0)


def test_attention_repeat_and_graph_replay(gb, oracle, cuda):
    """Several positions in a row through one workspace (the tickets re-arm),
    captured in a CUDA graph whose position comes from device memory."""
    nh, nkv, hd, ms = 8, 2, 128, 600
    kc = oracle.synth_normal(nkv * ms * hd, 9, 4)
    vc = oracle.synth_normal(nkv * ms * hd, 9, 5)
    dkc, dvc = to_dev(cuda, kc), to_dev(cuda, vc)
    cs = cuda.empty(ms * hd, dtype=cuda.float32, device="cuda")
    gb.rope_table(cs, ms, hd)
    ws = cuda.zeros(gb.attn_workspace_bytes(nh, nkv, hd, ms), dtype=cuda.uint8, device="cuda")
    d_pos = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    dq = cuda.zeros(nh * hd, dtype=cuda.float32, device="cuda")
    dk = cuda.zeros(nkv * hd, dtype=cuda.float32, device="cuda")
    dv = cuda.zeros(nkv * hd, dtype=cuda.float32, device="cuda")
    out = cuda.zeros(nh * hd, dtype=cuda.float32, device="cuda")
    s = cuda.cuda.Stream()
    g = cuda.cuda.CUDAGraph()
    with cuda.cuda.stream(s):
        gb.attention_decode(dq, dk, dv, dkc, dvc, cs, d_pos, nh, nkv, hd, ms, out, ws, stream=s.cuda_stream)
    s.synchronize()
    with cuda.cuda.graph(g, stream=s):
        gb.attention_decode(dq, dk, dv, dkc, dvc, cs, d_pos, nh, nkv, hd, ms, out, ws, stream=s.cuda_stream)
    kc_h, vc_h = kc.copy(), vc.copy()
    for pos in (0, 100, 101, 257, 599):
        q = oracle.synth_normal(nh * hd, pos, 1)
        k = oracle.synth_normal(nkv * hd, pos, 2)
        v = oracle.synth_normal(nkv * hd, pos, 3)
        dq.copy_(to_dev(cuda, q)); dk.copy_(to_dev(cuda, k)); dv.copy_(to_dev(cuda, v))
        d_pos.fill_(pos)
        cuda.cuda.synchronize()
        g.replay()
        cuda.cuda.synchronize()
        o_ref, kc_h, vc_h = oracle.attention_step(q, k, v, kc_h, vc_h, nh, nkv, hd, ms, pos)
        assert rel_l2(from_dev(out), o_ref) <= 1e-5, pos
    assert np.array_equal(from_dev(dkc), kc_h)
    assert np.array_equal(from_dev(dvc), vc_h)


def test_attention_position_out_of_range(gb, oracle, cuda):
    """pos >= max_seq (the reference asserts, engine.c:422): the kernel sets
    its error word and writes nothing."""
    nh, nkv, hd, ms = 8, 2, 64, 32
    kc = oracle.synth_normal(nkv * ms * hd, 1, 4)
    vc = oracle.synth_normal(nkv * ms * hd, 1, 5)
    q = oracle.synth_normal(nh * hd, 1, 1)
    k = oracle.synth_normal(nkv * hd, 1, 2)
    v = oracle.synth_normal(nkv * hd, 1, 3)
    _, kc_g, vc_g, ws = run_attention(gb, cuda, q, k, v, kc, vc, nh, nkv, hd, ms, ms)
    assert np.array_equal(kc_g, kc) and np.array_equal(vc_g, vc)
    err = from_dev(ws).view(np.uint32)[-1]
    assert err == 4   # -GB_EPOS
