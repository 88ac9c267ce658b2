"""gb_attention_decode_static: the split-K attention entry point whose scratch
is a static device array (no workspace argument, no allocation).  Compared
with gb_attention_decode on two calls in a row; runs alone or after every
other test (the scratch's tickets must be back at zero after each call)."""
import numpy as np
import pytest

from helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu


def _setup(oracle, cuda, nh, nkv, hd, ms, seed):
    t = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    kc = oracle.synth_normal(nkv * ms * hd, seed, 4)
    vc = oracle.synth_normal(nkv * ms * hd, seed, 5)
    return t, kc, vc


@pytest.mark.parametrize("nh,nkv,hd,ms,pos", [(8, 2, 128, 300, 257), (32, 8, 128, 8448, 8192), (4, 4, 64, 40, 3)])
def test_static_matches_workspace_entry(gb, oracle, cuda, nh, nkv, hd, ms, pos):
    t, kc, vc = _setup(oracle, cuda, nh, nkv, hd, ms, 17)
    cs = cuda.empty(ms * hd, dtype=cuda.float32, device="cuda")
    gb.rope_table(cs, ms, hd)
    ws = cuda.zeros(gb.attn_workspace_bytes(nh, nkv, hd, ms), dtype=cuda.uint8, device="cuda")
    kc_a, vc_a, kc_b, vc_b = t(kc), t(vc), t(kc), t(vc)
    for step in range(2):   # two calls in a row, positions pos and pos + 1
        p = pos + step
        q = oracle.synth_normal(nh * hd, 30 + step, 1)
        k = oracle.synth_normal(nkv * hd, 30 + step, 2)
        v = oracle.synth_normal(nkv * hd, 30 + step, 3)
        d_pos = cuda.tensor([p], dtype=cuda.int32, device="cuda")
        out_a = cuda.empty(nh * hd, dtype=cuda.float32, device="cuda")
        out_b = cuda.empty(nh * hd, dtype=cuda.float32, device="cuda")
        gb.attention_decode(t(q), t(k), t(v), kc_a, vc_a, cs, d_pos, nh, nkv, hd, ms, out_a, ws)
        gb.attention_decode_static(t(q), t(k), t(v), kc_b, vc_b, cs, d_pos, nh, nkv, hd, ms, out_b)
        cuda.cuda.synchronize()
        # same kernel, same split geometry: identical bits
        assert cuda.equal(out_a, out_b), step
        assert cuda.equal(kc_a, kc_b) and cuda.equal(vc_a, vc_b)
    assert gb.lib().gb_attention_static_error(1) == 0


def test_static_against_oracle_and_limits(gb, oracle, cuda):
    nh, nkv, hd, ms, pos = 8, 2, 128, 300, 120
    t, kc, vc = _setup(oracle, cuda, nh, nkv, hd, ms, 23)
    q, k, v = (oracle.synth_normal(n, 23, i) for i, n in ((1, nh * hd), (2, nkv * hd), (3, nkv * hd)))
    o_ref, kc_ref, _ = oracle.attention_step(q, k, v, kc, vc, nh, nkv, hd, ms, pos)
    cs = cuda.empty(ms * hd, dtype=cuda.float32, device="cuda")
    gb.rope_table(cs, ms, hd)
    dkc, dvc = t(kc), t(vc)
    out = cuda.empty(nh * hd, dtype=cuda.float32, device="cuda")
    gb.attention_decode_static(t(q), t(k), t(v), dkc, dvc, cs, cuda.tensor([pos], dtype=cuda.int32, device="cuda"),
                               nh, nkv, hd, ms, out)
    cuda.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), o_ref) <= REL_L2_TOL
    assert np.array_equal(dkc.cpu().numpy(), kc_ref)
    L = gb.lib()
    # more KV heads than the static scratch has ticket words is refused (the
    # split partials are bounded by one CTA per SM, so they always fit)
    assert L.gb_attention_decode_static(out.data_ptr(), out.data_ptr(), out.data_ptr(), dkc.data_ptr(),
                                        dvc.data_ptr(), cs.data_ptr(), out.data_ptr(), 2048, 1024, 128, ms,
                                        out.data_ptr(), None) == gb.GB_ELIMIT
    # a position outside [0, max_seq) lands in the static error word
    gb.attention_decode_static(t(q), t(k), t(v), dkc, dvc, cs, cuda.tensor([ms], dtype=cuda.int32, device="cuda"),
                               nh, nkv, hd, ms, out)
    cuda.cuda.synchronize()
    assert L.gb_attention_static_error(1) == gb.GB_EPOS
    assert L.gb_attention_static_error(0) == 0
