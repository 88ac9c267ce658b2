"""The drop-in inside the reference engine: src/engine/engine.c compiled with
-DUSE_CUDA=1 and linked against libguanaco_b200.so (oracle/_ref/libref_dropin.so,
built by oracle/Makefile from the reference sources).  Its forward() takes the
cuda_transformer_layer_gpu branch of transformer_layer (engine.c:314-350) for
every layer, back to back with no cuda_finish_layer between them, and the
output head goes through the vtable slot of backend_create(AUTO)
(engine.c:590).  The same engine compiled without USE_CUDA (libref.so) runs
the same seeded model on the CPU; logits must agree within 1e-3 relative L2.
Prompts of T > 1 tokens take the engine's CPU prefill, whose K / V rows
reach the device through cuda_sync_kv_cache (engine.c:394-403)."""
import os

import numpy as np
import pytest

from tests.helpers import REL_L2_TOL, rel_l2
from tests.synth_model import fill_kv, gpu_blocks, synth_model

pytestmark = pytest.mark.gpu

SEED = 4242


def _pair(gb, oracle, cuda, H, nh, nkv, n_layers, ff, vocab, max_seq):
    if not (oracle.ref_available() and oracle.dropin_available()):
        pytest.skip("oracle/_ref/libref.so or libref_dropin.so not built")
    gb.lib()
    threads = os.cpu_count() or 1
    oracle.ref().ref_set_threads(threads)
    m = synth_model(oracle, H, nh, nkv, n_layers, ff, vocab, max_seq, SEED, gen=gpu_blocks(gb, cuda))
    cpu = oracle.RefModel(m)
    eng = oracle.RefModel(m, lib=oracle.dropin())
    eng.to_gpu(threads)
    return m, cpu, eng


def _close(oracle, *models):
    for x in models:
        x.close()
    oracle.ref().ref_set_threads(1)


def test_engine_forward_through_dropin_llama8b_width(gb, oracle, cuda):
    """Llama-3.1-8B width (hidden 4096, 32 / 8 heads, FFN 14336, the full
    128256-row output head), two layers, K / V filled to 4096 positions on
    the host (the drop-in uploads what it has not computed), four greedy
    steps through the unchanged engine."""
    ctx = 4096
    m, cpu, eng = _pair(gb, oracle, cuda, 4096, 32, 8, 2, 14336, 128256, ctx + 8)
    try:
        fill_kv(oracle, cpu, m, ctx, SEED)
        fill_kv(oracle, eng, m, ctx, SEED)
        token, agree = 1, 0
        for pos in range(ctx, ctx + 4):
            lc = cpu.forward(token, pos)
            lg = eng.forward(token, pos)
            assert rel_l2(lg, lc) <= REL_L2_TOL, pos
            nc, ng = oracle.argmax(lc), oracle.argmax(lg)
            s = np.sort(lc)
            if s[-1] - s[-2] > 1e-3 * max(1.0, abs(float(s[-1]))):
                assert nc == ng, pos
                agree += 1
            token = nc
        assert agree >= 2
        # the appended rows reached the engine's host cache (session files
        # and the prompt cache read it)
        kv = m.n_kv * m.max_seq * m.hd
        for layer in range(m.n_layers):
            for which in (0, 1):
                a = cpu.kv(layer, which, kv).reshape(m.n_kv, m.max_seq, m.hd)[:, ctx:ctx + 4]
                b = eng.kv(layer, which, kv).reshape(m.n_kv, m.max_seq, m.hd)[:, ctx:ctx + 4]
                assert rel_l2(b, a) <= REL_L2_TOL
    finally:
        _close(oracle, eng, cpu)


def test_engine_prefill_on_cpu_then_decode_through_dropin(gb, oracle, cuda):
    """A 12-token prompt takes the engine's T > 1 CPU path (its K / V rows
    reach the device through cuda_sync_kv_cache), then 10 greedy decode
    steps run through the drop-in layer and the vtable output head."""
    m, cpu, eng = _pair(gb, oracle, cuda, 2048, 16, 4, 3, 4096, 3000, 64)
    try:
        prompt = np.random.RandomState(SEED).randint(0, m.vocab, 12)
        lc = cpu.forward_tokens(prompt, 0)
        lg = eng.forward_tokens(prompt, 0)
        assert rel_l2(lg, lc) <= REL_L2_TOL
        token = oracle.argmax(lc)
        for pos in range(len(prompt), len(prompt) + 10):
            lc = cpu.forward(token, pos)
            lg = eng.forward(token, pos)
            assert rel_l2(lg, lc) <= REL_L2_TOL, pos
            token = oracle.argmax(lc)
    finally:
        _close(oracle, eng, cpu)
