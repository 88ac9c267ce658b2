"""Prefill on the device (gb_model_prefill): a prompt of T tokens through
every layer at once -- tensor-core GEMMs, RoPE + KV append, causal attention
-- against the reference forward() over the same prompt
(src/engine/engine.c:559-594 with n_tokens = T, the reference's CPU prefill,
compiled unchanged into oracle/_ref/libref.so) on the same seeded weights.

* gb_prefill_attention against an fp64 causal softmax (bound 1e-5 relative
  L2: fp32 arithmetic, only the summation order differs).
* Whole models: last-row logits within the 1e-3 relative-L2 bound, the same
  greedy token wherever the reference's top two logits differ by more than
  1e-3 relative, every layer's K / V cache rows within 1e-4 of the
  reference's, and decode continuing from the prefilled cache.
* A prompt split into two prefills (pos > 0), and chunked prefill
  (GB_PREFILL_CHUNK), against one reference prefill.
* The Llama-3.1-8B width (two layers, the full output head, a 300-token
  prompt) against the reference forward()."""
import os

import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, read_device, rel_l2, to_dev, from_dev
from tests.synth_model import gpu_blocks, synth_model

pytestmark = pytest.mark.gpu

SEED = 1234


def _attn_fp64(q, kc, vc, T, pos, nh, nkv, hd):
    G = nh // nkv
    out = np.zeros((T, nh * hd))
    qpos = pos + np.arange(T)
    for h in range(nh):
        g = h // G
        Q = q[:, h * hd:(h + 1) * hd].astype(np.float64)
        K = kc[g, :pos + T].astype(np.float64)
        V = vc[g, :pos + T].astype(np.float64)
        S = Q @ K.T / np.sqrt(hd)
        S[np.arange(pos + T)[None, :] > qpos[:, None]] = -np.inf
        S -= S.max(1, keepdims=True)
        P = np.exp(S)
        P /= P.sum(1, keepdims=True)
        out[:, h * hd:(h + 1) * hd] = P @ V
    return out


@pytest.mark.parametrize("T,pos,nh,nkv,hd,max_seq", [
    (1, 0, 8, 2, 128, 64), (37, 0, 32, 8, 128, 256), (130, 5, 8, 8, 64, 200), (64, 100, 16, 2, 64, 300),
    (200, 0, 32, 8, 128, 256), (9, 20, 8, 1, 128, 64), (70, 3, 32, 4, 64, 80)])
def test_prefill_attention_matches_fp64(gb, oracle, cuda, T, pos, nh, nkv, hd, max_seq):
    q = oracle.synth_normal(T * nh * hd, 11, T).reshape(T, nh * hd)
    kc = oracle.synth_normal(nkv * max_seq * hd, 11, 1).reshape(nkv, max_seq, hd)
    vc = oracle.synth_normal(nkv * max_seq * hd, 11, 2).reshape(nkv, max_seq, hd)
    out = cuda.full((T, nh * hd), float("nan"), dtype=cuda.float32, device="cuda")
    gb.prefill_attention(to_dev(cuda, q), to_dev(cuda, kc), to_dev(cuda, vc), out, T, pos, nh, nkv, hd, max_seq)
    cuda.cuda.synchronize()
    got = from_dev(out)
    ref = _attn_fp64(q, kc, vc, T, pos, nh, nkv, hd)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-5, rel_l2(got, ref)
    for t in (0, T - 1):   # single rows too (the first query sees one key at pos 0)
        assert rel_l2(got[t], ref[t]) <= 1e-5


def test_prefill_attention_rejects_past_max_seq(gb, cuda):
    q = cuda.zeros(4 * 8 * 64, device="cuda")
    kc = cuda.zeros(2 * 16 * 64, device="cuda")
    with pytest.raises(gb.GBError):
        gb.prefill_attention(q, kc, kc, q, 4, 13, 8, 2, 64, 16)


def _models(gb, oracle, cuda, H, nh, nkv, n_layers, ff, vocab, max_seq):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    oracle.ref().ref_set_threads(os.cpu_count() or 1)
    m = synth_model(oracle, H, nh, nkv, n_layers, ff, vocab, max_seq, SEED, gen=gpu_blocks(gb, cuda))
    ref = oracle.RefModel(m)
    dm = gb.DecodeModel(H, nh, nkv, n_layers, ff, vocab, max_seq)
    dm.synthesize(SEED)
    return m, ref, dm


def _clear_winner(logits):
    s = np.sort(logits)
    return s[-1] - s[-2] > 1e-3 * max(1.0, abs(float(s[-1])))


def _check_logits(oracle, lg, lr, nxt):
    assert rel_l2(lg, lr) <= REL_L2_TOL, rel_l2(lg, lr)
    if _clear_winner(lr):
        assert nxt == oracle.argmax(lr)


def _check_kv(m, ref, dm, n):
    for l in range(m.n_layers):
        for which in (0, 1):
            ptr = dm.v_cache(l) if which else dm.k_cache(l)
            got = read_device(ptr, m.n_kv * m.max_seq * m.hd).reshape(m.n_kv, m.max_seq, m.hd)[:, :n]
            want = ref.kv(l, which, m.n_kv * m.max_seq * m.hd).reshape(m.n_kv, m.max_seq, m.hd)[:, :n]
            assert rel_l2(got, want) <= 1e-4, (l, which, rel_l2(got, want))


# (H, heads, kv heads, layers, FFN, vocabulary, max_seq): head_dim 64 with
# groups of 4, head_dim 128 with groups of 2, and TinyLlama-1.1B (22 layers,
# 32 / 4 heads of 64, FFN 5632, vocabulary 32000)
MODELS = {
    "hd64": (512, 8, 2, 4, 1536, 4096, 256),
    "hd128": (1024, 8, 4, 3, 2816, 8192, 256),
    "tinyllama": (2048, 32, 4, 22, 5632, 32000, 256),
    "hd64_long": (512, 8, 2, 2, 1536, 4096, 512),
}
PROMPT = {"hd64_long": 400}   # several 128-token tiles of every GEMM and attention block


@pytest.mark.parametrize("name", list(MODELS))
def test_prefill_matches_reference_forward(gb, oracle, cuda, name):
    m, ref, dm = _models(gb, oracle, cuda, *MODELS[name])
    try:
        prompt = np.random.RandomState(SEED).randint(0, m.vocab, PROMPT.get(name, 128)).astype(np.int32)
        lr = ref.forward_tokens(prompt, 0)
        lg = np.zeros(m.vocab, np.float32)
        nxt = dm.prefill_host(prompt, 0, lg)
        _check_logits(oracle, lg, lr, nxt)
        _check_kv(m, ref, dm, len(prompt))
        # decode continues from the prefilled cache
        token = oracle.argmax(lr)
        for pos in range(len(prompt), len(prompt) + 3):
            lr = ref.forward(int(token), pos)
            lg = np.zeros(m.vocab, np.float32)
            nxt = dm.decode_host(int(token), pos, lg)
            _check_logits(oracle, lg, lr, nxt)
            token = oracle.argmax(lr)
        assert dm.error() == 0
    finally:
        dm.close()
        ref.close()
        oracle.ref().ref_set_threads(1)


def test_prefill_in_two_parts_and_chunked(gb, oracle, cuda, monkeypatch):
    """70 tokens at position 0, then 58 at position 70 (the second attends to
    the first's cache), and the same prompt in chunks of 48: both against one
    reference prefill of all 128."""
    m, ref, dm = _models(gb, oracle, cuda, *MODELS["hd64"])
    try:
        prompt = np.random.RandomState(SEED + 1).randint(0, m.vocab, 128).astype(np.int32)
        lr = ref.forward_tokens(prompt, 0)
        dm.prefill_host(prompt[:70], 0)
        lg = np.zeros(m.vocab, np.float32)
        nxt = dm.prefill_host(prompt[70:], 70, lg)
        _check_logits(oracle, lg, lr, nxt)
        _check_kv(m, ref, dm, len(prompt))
        monkeypatch.setenv("GB_PREFILL_CHUNK", "48")
        lg2 = np.zeros(m.vocab, np.float32)
        nxt2 = dm.prefill_host(prompt, 0, lg2)
        _check_logits(oracle, lg2, lr, nxt2)
        _check_kv(m, ref, dm, len(prompt))
        assert dm.error() == 0
    finally:
        dm.close()
        ref.close()
        oracle.ref().ref_set_threads(1)


def test_prefill_device_entry_and_errors(gb, oracle, cuda):
    """The device entry point (tokens, logits and next token in HBM) gives the
    host entry's result; a prompt past max_seq is refused (GB_EPOS) and an
    out-of-vocabulary token sets the model's error word."""
    H, nh, nkv, L, ff, vocab, max_seq = MODELS["hd64"]
    dm = gb.DecodeModel(H, nh, nkv, L, ff, vocab, max_seq)
    try:
        dm.synthesize(SEED)
        prompt = np.random.RandomState(7).randint(0, vocab, 40).astype(np.int32)
        lh = np.zeros(vocab, np.float32)
        nh_ = dm.prefill_host(prompt, 0, lh)
        d_tok = to_dev(cuda, prompt)
        d_lg = cuda.zeros(vocab, device="cuda")
        d_next = cuda.zeros(1, dtype=cuda.int32, device="cuda")
        dm.prefill(d_tok, len(prompt), 0, d_lg, d_next)
        cuda.cuda.synchronize()
        assert int(from_dev(d_next)[0]) == nh_
        assert np.array_equal(from_dev(d_lg), lh)   # same launches, same bits
        with pytest.raises(gb.GBError):
            dm.prefill_host(prompt, max_seq - 10)
        bad = prompt.copy()
        bad[5] = vocab
        with pytest.raises(gb.GBError):
            dm.prefill_host(bad, 0)
    finally:
        dm.close()


def test_prefill_llama8b_width_matches_reference_forward(gb, oracle, cuda):
    """The benchmarked shapes: hidden 4096, 32 / 8 heads of 128, FFN 14336, the
    full 128256-row Q6_K output head, two layers, a 300-token prompt (gate /
    up on 256-token tiles, ffn_down at K = 14336), against the reference
    forward() over the same prompt; then two decode steps from the prefilled
    cache."""
    m, ref, dm = _models(gb, oracle, cuda, 4096, 32, 8, 2, 14336, 128256, 320)
    try:
        prompt = np.random.RandomState(SEED + 2).randint(0, m.vocab, 300).astype(np.int32)
        lr = ref.forward_tokens(prompt, 0)
        lg = np.zeros(m.vocab, np.float32)
        nxt = dm.prefill_host(prompt, 0, lg)
        _check_logits(oracle, lg, lr, nxt)
        _check_kv(m, ref, dm, len(prompt))
        token = oracle.argmax(lr)
        for pos in range(len(prompt), len(prompt) + 2):
            lr = ref.forward(int(token), pos)
            lg = np.zeros(m.vocab, np.float32)
            nxt = dm.decode_host(int(token), pos, lg)
            _check_logits(oracle, lg, lr, nxt)
            token = oracle.argmax(lr)
        assert dm.error() == 0
    finally:
        dm.close()
        ref.close()
        oracle.ref().ref_set_threads(1)
