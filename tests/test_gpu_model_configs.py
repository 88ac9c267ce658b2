"""Whole-model parity at the benchmarked shapes: the device decode step (every
launch the benchmark times) against the reference forward() compiled
unchanged from the reference sources (oracle/_ref/libref.so,
src/engine/engine.c:559-594), on the same seeded weights and caches.

* Llama-3.1-8B width (config 4): hidden 4096, 32 / 8 heads, FFN 14336, the
  full 128256-row Q6_K output head, two layers, K / V filled to 4096
  positions, four teacher-forced steps.
* TinyLlama-1.1B (config 3): all 22 layers (hidden 2048, 32 / 4 heads,
  FFN 5632, vocabulary 32000), a 128-token prompt through the decode path,
  then eight teacher-forced greedy steps.

Logits must agree within the 1e-3 relative-L2 bound; the greedy token must
agree wherever the reference's top two logits differ by more than 1e-3
relative (teacher forcing keeps both sides on the reference's tokens)."""
import os

import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, rel_l2
from tests.synth_model import fill_kv, gpu_blocks, synth_model

pytestmark = pytest.mark.gpu

SEED = 1234


def _clear_winner(logits):
    s = np.sort(logits)
    return s[-1] - s[-2] > 1e-3 * max(1.0, abs(float(s[-1])))


def _step(oracle, ref, dm, vocab, token, pos):
    lr = ref.forward(token, pos)
    lg = np.zeros(vocab, np.float32)
    nxt = dm.decode_host(token, pos, lg)
    err = rel_l2(lg, lr)
    assert err <= REL_L2_TOL, (pos, err)
    tok_ref = oracle.argmax(lr)
    agreed = None
    if _clear_winner(lr):
        assert nxt == tok_ref, (pos, nxt, tok_ref)
        agreed = True
    return tok_ref, err, agreed


def _models(gb, oracle, cuda, H, nh, nkv, n_layers, ff, vocab, max_seq):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    oracle.ref().ref_set_threads(os.cpu_count() or 1)
    m = synth_model(oracle, H, nh, nkv, n_layers, ff, vocab, max_seq, SEED, gen=gpu_blocks(gb, cuda))
    ref = oracle.RefModel(m)
    dm = gb.DecodeModel(H, nh, nkv, n_layers, ff, vocab, max_seq)
    dm.synthesize(SEED)
    return m, ref, dm


def test_llama8b_width_matches_reference_forward(gb, oracle, cuda):
    ctx = 4096
    m, ref, dm = _models(gb, oracle, cuda, 4096, 32, 8, 2, 14336, 128256, ctx + 8)
    try:
        fill_kv(oracle, ref, m, ctx, SEED)
        dm.fill_kv(ctx, SEED)
        token, agree, worst = 1, 0, 0.0
        for pos in range(ctx, ctx + 4):
            token, err, ok = _step(oracle, ref, dm, m.vocab, token, pos)
            worst = max(worst, err)
            agree += bool(ok)
        assert dm.error() == 0
        assert agree >= 2
    finally:
        dm.close()
        ref.close()
        oracle.ref().ref_set_threads(1)


def test_tinyllama_22_layers_prompt_then_greedy(gb, oracle, cuda):
    m, ref, dm = _models(gb, oracle, cuda, 2048, 32, 4, 22, 5632, 32000, 256)
    try:
        prompt = np.random.RandomState(SEED).randint(0, m.vocab, 128)
        agree = 0
        for pos, tok in enumerate(prompt):
            lr = ref.forward(int(tok), pos)
            lg = np.zeros(m.vocab, np.float32)
            dm.decode_host(int(tok), pos, lg)
            assert rel_l2(lg, lr) <= REL_L2_TOL, pos
        token = oracle.argmax(lr)
        for pos in range(len(prompt), len(prompt) + 8):
            token, _, ok = _step(oracle, ref, dm, m.vocab, token, pos)
            agree += bool(ok)
        assert dm.error() == 0
        assert agree >= 4
    finally:
        dm.close()
        ref.close()
        oracle.ref().ref_set_threads(1)
