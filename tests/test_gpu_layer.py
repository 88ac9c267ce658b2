"""GPU parity of a whole decode layer through the drop-in
cuda_transformer_layer_gpu (src/kernels/cuda/cuda_layer_kernels.cu:605), and
of the device-resident decode model against the reference forward()
(engine.c:559-594, compiled from the reference sources into oracle/_ref)."""
import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu


def layer_weights(oracle, H, nh, nkv, hd, ff, seed, dtypes=(4, 4, 5, 4, 4, 4, 5)):
    kv = nkv * hd
    shapes = [(nh * hd, H), (kv, H), (kv, H), (H, nh * hd), (ff, H), (ff, H), (H, ff)]
    ws = [oracle.synth_blocks(dt, r, c, seed, 10 + i) for i, (dt, (r, c)) in enumerate(zip(dtypes, shapes))]
    ra = (1.0 + 0.01 * oracle.synth_normal(H, seed, 30)).astype(np.float32)
    rf = (1.0 + 0.01 * oracle.synth_normal(H, seed, 31)).astype(np.float32)
    return ws, list(dtypes), shapes, ra, rf


@pytest.mark.parametrize("H,nh,nkv,ff,dtypes", [
    (512, 4, 2, 1024, (4, 4, 5, 4, 4, 4, 5)),
    (512, 8, 2, 1536, (4, 4, 4, 4, 4, 4, 4)),
    (1024, 8, 8, 768, (2, 2, 2, 2, 2, 2, 2)),
    # every matrix on the TMA path (Q6_K rows of 8-block multiples): RMSNorm and
    # the SwiGLU product run inside the matvecs
    (2048, 16, 4, 4096, (4, 4, 5, 4, 4, 4, 5)),
])
def test_dropin_layer_sequence(gb, oracle, cuda, H, nh, nkv, ff, dtypes):
    hd = H // nh
    ms = 40
    layer = 7
    ws, dts, shapes, ra, rf = layer_weights(oracle, H, nh, nkv, hd, ff, 99, dtypes)
    L = gb.lib()
    dptr = [L.cuda_upload_weight(w.ctypes.data, w.nbytes) for w in ws]
    assert all(dptr)
    # host KV as kv_cache_create lays it out for one layer; positions [0, 9)
    # come from an earlier (CPU) prefill
    kc = np.zeros(nkv * ms * hd, np.float32)
    vc = np.zeros(nkv * ms * hd, np.float32)
    kc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 5, 1).reshape(nkv, 9, hd)
    vc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 5, 2).reshape(nkv, 9, hd)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    h = oracle.synth_normal(H, 5, 3)
    h_ref = h.copy()
    for pos in range(9, 14):
        args = []
        for d, (r, c), dt in zip(dptr, shapes, dts):
            args += [d, r, c, dt]
        rc = L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data,
                                          kc.ctypes.data, vc.ctypes.data, ms * hd, H, nh, nkv, hd, pos, layer, ms)
        assert rc == 0
        L.cuda_finish_layer()
        h_ref, kc_ref, vc_ref = oracle.layer_decode(ws, dts, shapes, ra, rf, h_ref, kc_ref, vc_ref,
                                                     H, nh, nkv, hd, ff, ms, pos)
        assert rel_l2(h, h_ref) <= REL_L2_TOL, pos
        # the appended row was written back into the host cache
        row = lambda a: a.reshape(nkv, ms, hd)[:, pos]  # noqa: E731
        assert rel_l2(row(kc), row(kc_ref)) <= REL_L2_TOL
        assert rel_l2(row(vc), row(vc_ref)) <= REL_L2_TOL
        h = h_ref.copy()   # teacher-force the next step from the oracle state
        kc[:] = kc_ref
        vc[:] = vc_ref
        L.cuda_sync_kv_cache(layer, nkv, hd, pos, 1, kc.ctypes.data, vc.ctypes.data, ms * hd, ms)
    # out-of-range position falls back to the caller (non-zero return)
    args = []
    for d, (r, c), dt in zip(dptr, shapes, dts):
        args += [d, r, c, dt]
    assert L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data, kc.ctypes.data,
                                        vc.ctypes.data, ms * hd, H, nh, nkv, hd, ms, layer, ms) == gb.GB_EPOS


class TinyModel:
    def __init__(self, oracle, H=256, nh=4, nkv=2, ff=512, vocab=1000, n_layers=2, max_seq=64, seed=7):
        self.H, self.n_heads, self.n_kv, self.hd, self.ff = H, nh, nkv, H // nh, ff
        self.vocab, self.n_layers, self.max_seq = vocab, n_layers, max_seq

        class Lw:
            pass
        self.layers = []
        for l in range(n_layers):
            ws, dts, shapes, ra, rf = layer_weights(oracle, H, nh, nkv, H // nh, ff, seed * 100 + l)
            lw = Lw()
            lw.w, lw.dtypes, lw.shapes, lw.rms_att, lw.rms_ffn = ws, dts, shapes, ra, rf
            self.layers.append(lw)
        self.emb_dtype, self.lm_dtype = 4, 5
        self.embedding = oracle.synth_blocks(4, vocab, H, seed, 900)
        self.lm_head = oracle.synth_blocks(5, vocab, H, seed, 901)
        self.rms_final = (1.0 + 0.01 * oracle.synth_normal(H, seed, 902)).astype(np.float32)


def upload(cuda, arr):
    t = cuda.zeros(arr.nbytes + 16, dtype=cuda.uint8, device="cuda")
    t[: arr.nbytes] = cuda.from_numpy(arr.view(np.uint8).ravel()).cuda()
    return t


@pytest.mark.parametrize("shape", [
    # rows too short for the Q6_K tensor maps: one launch per matrix
    dict(H=256, nh=4, nkv=2, ff=512, vocab=1000),
    # every matrix on the TMA path, grouped launches
    dict(H=2048, nh=16, nkv=4, ff=4096, vocab=1000),
])
def test_model_decode_matches_reference_forward(gb, oracle, cuda, shape):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    m = TinyModel(oracle, **shape)
    ref = oracle.RefModel(m)
    dm = gb.DecodeModel(m.H, m.n_heads, m.n_kv, m.n_layers, m.ff, m.vocab, m.max_seq)
    keep = []
    try:
        for l, lw in enumerate(m.layers):
            for i, (w, dt) in enumerate(zip(lw.w, lw.dtypes)):
                t = upload(cuda, w)
                keep.append(t)
                dm.set_matrix(l, i, dt, t)
            ra, rf = upload(cuda, lw.rms_att), upload(cuda, lw.rms_ffn)
            keep += [ra, rf]
            dm.set_norms(l, ra, rf)
        e, lm, rfin = upload(cuda, m.embedding), upload(cuda, m.lm_head), upload(cuda, m.rms_final)
        keep += [e, lm, rfin]
        dm.set_head(4, e, rfin, 5, lm)
        token = 17
        agree = 0
        for pos in range(12):
            logits_ref = ref.forward(token, pos)
            logits = np.zeros(m.vocab, np.float32)
            nxt = dm.decode_host(token, pos, logits)
            assert rel_l2(logits, logits_ref) <= REL_L2_TOL, pos
            tok_ref = oracle.argmax(logits_ref)
            srt = np.sort(logits_ref)
            if srt[-1] - srt[-2] > 1e-3 * max(1.0, abs(srt[-1])):
                assert nxt == tok_ref, pos
                agree += 1
            token = tok_ref   # teacher forcing on the reference's choice
        assert agree >= 8
    finally:
        dm.close()
        ref.close()


def test_model_synthesized_decode_runs(gb, cuda):
    """Synthetic Q4_K_M-style model: greedy decode produces valid tokens and
    replays the captured graph deterministically."""
    dm = gb.DecodeModel(512, 4, 2, 3, 1024, 2048, 128)
    try:
        dm.synthesize(1234)
        toks = []
        t = 1
        for pos in range(20):
            t = dm.decode_host(t, pos)
            assert 0 <= t < 2048
            toks.append(t)
        dm2 = gb.DecodeModel(512, 4, 2, 3, 1024, 2048, 128)
        dm2.synthesize(1234)
        t = 1
        for pos in range(20):
            t = dm2.decode_host(t, pos)
            assert t == toks[pos]
        dm2.close()
        with pytest.raises(gb.GBError):
            dm.decode_host(1, 128)
    finally:
        dm.close()


@pytest.mark.parametrize("vocab", [20000, 4096 * 3 + 5])
def test_model_argmax_split_first_maximum(gb, cuda, vocab):
    """The output head's argmax runs split over several CTAs for long
    vocabularies; the next token is the first index of the maximum logit."""
    dm = gb.DecodeModel(256, 4, 2, 1, 512, vocab, 32)
    try:
        dm.synthesize(77)
        for pos in range(3):
            logits = np.zeros(vocab, np.float32)
            nxt = dm.decode_host(5 + pos, pos, logits=logits)
            assert nxt == int(np.argmax(logits))
    finally:
        dm.close()


def test_dropin_layer_rewind_uses_restored_host_kv(gb, oracle, cuda):
    """After decoding positions 9..12 on the GPU, the engine restores another
    session (new host K/V for positions 0..8, session.c kv_cache_load) and
    decodes position 9 again: the layer must attend over the restored values,
    not the device copy of the old conversation."""
    H, nh, nkv, ff, ms, layer = 512, 8, 2, 1536, 40, 13
    hd = H // nh
    ws, dts, shapes, ra, rf = layer_weights(oracle, H, nh, nkv, hd, ff, 21, (4, 4, 4, 4, 4, 4, 4))
    L = gb.lib()
    dptr = [L.cuda_upload_weight(w.ctypes.data, w.nbytes) for w in ws]
    args = []
    for d, (r, c), dt in zip(dptr, shapes, dts):
        args += [d, r, c, dt]
    kc = np.zeros(nkv * ms * hd, np.float32)
    vc = np.zeros(nkv * ms * hd, np.float32)
    kc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 31, 1).reshape(nkv, 9, hd)
    vc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 31, 2).reshape(nkv, 9, hd)
    for pos in range(9, 13):   # the first conversation, decoded on the GPU
        h = oracle.synth_normal(H, 40 + pos, 3)
        assert L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data, kc.ctypes.data,
                                            vc.ctypes.data, ms * hd, H, nh, nkv, hd, pos, layer, ms) == 0
        L.cuda_finish_layer()
    # restore another session: new K/V for positions 0..8 in the host cache
    kc[:] = 0.0
    vc[:] = 0.0
    kc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 32, 1).reshape(nkv, 9, hd)
    vc.reshape(nkv, ms, hd)[:, :9] = oracle.synth_normal(nkv * 9 * hd, 32, 2).reshape(nkv, 9, hd)
    h = oracle.synth_normal(H, 77, 3)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    h_ref, _, _ = oracle.layer_decode(ws, dts, shapes, ra, rf, h.copy(), kc_ref, vc_ref, H, nh, nkv, hd, ff, ms, 9)
    assert L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data, kc.ctypes.data,
                                        vc.ctypes.data, ms * hd, H, nh, nkv, hd, 9, layer, ms) == 0
    L.cuda_finish_layer()
    assert rel_l2(h, h_ref) <= REL_L2_TOL


def test_dropin_layer_shape_change_rezeroes_attention_tickets(gb, oracle, cuda):
    """The drop-in context keeps one attention workspace; a later call with a
    smaller shape reuses it, and its split-merge tickets then fall on words
    that held the earlier shape's partials.  Both calls must match the
    reference layer."""
    L = gb.lib()
    for H, nh, nkv, ff, ms, pos, layer in ((512, 4, 2, 1024, 300, 200, 21), (512, 8, 2, 1536, 40, 9, 22)):
        hd = H // nh
        ws, dts, shapes, ra, rf = layer_weights(oracle, H, nh, nkv, hd, ff, 23, (4, 4, 4, 4, 4, 4, 4))
        dptr = [L.cuda_upload_weight(w.ctypes.data, w.nbytes) for w in ws]
        args = []
        for d, (r, c), dt in zip(dptr, shapes, dts):
            args += [d, r, c, dt]
        kc = np.zeros(nkv * ms * hd, np.float32)
        vc = np.zeros(nkv * ms * hd, np.float32)
        kc.reshape(nkv, ms, hd)[:, :pos] = oracle.synth_normal(nkv * pos * hd, 41, 1).reshape(nkv, pos, hd)
        vc.reshape(nkv, ms, hd)[:, :pos] = oracle.synth_normal(nkv * pos * hd, 41, 2).reshape(nkv, pos, hd)
        h = oracle.synth_normal(H, 43, 3)
        kc_ref, vc_ref = kc.copy(), vc.copy()
        h_ref, _, _ = oracle.layer_decode(ws, dts, shapes, ra, rf, h.copy(), kc_ref, vc_ref, H, nh, nkv, hd, ff, ms,
                                          pos)
        assert L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data, kc.ctypes.data,
                                            vc.ctypes.data, ms * hd, H, nh, nkv, hd, pos, layer, ms) == 0
        L.cuda_finish_layer()
        assert rel_l2(h, h_ref) <= REL_L2_TOL, (ms, pos)


def test_dropin_norm_cache_follows_host_values(gb, oracle, cuda):
    """Norm weights are cached by host pointer: new values at the same address
    (a freed and reallocated host buffer) must be used, not the old copy."""
    H, nh, nkv, ff, ms, layer = 512, 8, 2, 1536, 40, 11
    hd = H // nh
    ws, dts, shapes, ra, rf = layer_weights(oracle, H, nh, nkv, hd, ff, 5, (4, 4, 4, 4, 4, 4, 4))
    L = gb.lib()
    dptr = [L.cuda_upload_weight(w.ctypes.data, w.nbytes) for w in ws]
    kc = np.zeros(nkv * ms * hd, np.float32)
    vc = np.zeros(nkv * ms * hd, np.float32)
    args = []
    for d, (r, c), dt in zip(dptr, shapes, dts):
        args += [d, r, c, dt]
    for trial in range(2):
        if trial == 1:   # same arrays, new values
            ra[:] = (1.0 + 0.05 * oracle.synth_normal(H, 6, 30)).astype(np.float32)
            rf[:] = (1.0 + 0.05 * oracle.synth_normal(H, 6, 31)).astype(np.float32)
        h = oracle.synth_normal(H, 5, 3)
        kc_ref, vc_ref = kc.copy(), vc.copy()
        h_ref, _, _ = oracle.layer_decode(ws, dts, shapes, ra, rf, h.copy(), kc_ref, vc_ref, H, nh, nkv, hd, ff, ms, 0)
        assert L.cuda_transformer_layer_gpu(*args, ra.ctypes.data, rf.ctypes.data, h.ctypes.data, kc.ctypes.data,
                                            vc.ctypes.data, ms * hd, H, nh, nkv, hd, 0, layer, ms) == 0
        L.cuda_finish_layer()
        assert rel_l2(h, h_ref) <= REL_L2_TOL, trial
