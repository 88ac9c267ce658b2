"""Tensor-parallel decode on two GPUs: each rank holds its slice of the same
synthetic model (heads, FFN rows / columns, vocabulary rows), the ranks add
their partial hidden vectors over NVLink peer memory, and the greedy tokens
must match the one-GPU model; each rank's logits must match its slice of the
one-GPU logits.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# H 2048 keeps every matrix on the tensor-map path; ff 5120 gives each of two
# ranks 2560 FFN columns, so the Q6_K ffn_down shard needs zero padding
CFG = dict(hidden_dim=2048, n_heads=16, n_kv_heads=4, n_layers=2, ff_dim=5120, vocab_size=5000, max_seq=64)
# eight ranks: one KV head (two q heads) and 768 FFN rows per rank, as the
# Llama-3.1-8B shape gives at eight GPUs; 4096 positions of context so the
# attention of each rank's single KV head splits over many CTAs
CFG8 = dict(hidden_dim=2048, n_heads=16, n_kv_heads=8, n_layers=2, ff_dim=6144, vocab_size=5000, max_seq=4120)
CTX8 = 4096
SEED, CTX, STEPS = 4321, 20, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(dm, vocab_rows, ctx):
    toks, logits = [], []
    tok, pos = 7, ctx
    for _ in range(STEPS):
        lg = np.zeros(vocab_rows, np.float32)
        tok = dm.decode_host(tok, pos, logits=lg)
        toks.append(tok)
        logits.append(lg)
        pos += 1
    return toks, logits


def _worker(rank, world, port, q, fused, c, ctx, exchange):
    if not fused:
        os.environ["GB_TP_FUSED"] = "0"
    if exchange:
        os.environ["GB_TP_EXCHANGE"] = exchange
    import torch
    import torch.distributed as dist
    import guanaco_b200 as gb
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                            c["vocab_size"], c["max_seq"], tp_rank=rank, tp_world=world)
        dm.exchange_handles(dist)
        dm.synthesize(SEED)
        dm.fill_kv(ctx, SEED)
        _, _, off, n = dm.tp_info()
        toks, logits = _decode(dm, n, ctx)
        assert dm.error() == 0
        q.put((rank, off, toks, logits))
        dist.barrier()
        dm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,fused,big,exchange", [
    (2, True, False, "direct"), (2, True, False, "slice"), (2, False, False, None), (2, True, True, None),
    (4, True, False, None), (4, True, True, "slice"), (4, True, True, "direct"),
    (8, True, True, None), (8, False, True, None)])
def test_tp_decode_matches_one_gpu(gb, cuda, world, fused, big, exchange):
    """fused: the hidden-state exchanges run inside the wo / ffn_down matvecs
    (push) and the next RMSNorm matvec (sum), in the direct form (every CTA
    sums all ranks' slots) or the slice form (each CTA sums one slice, the
    CTAs meet on per-CTA flags); otherwise each exchange is its own
    all-reduce launch."""
    if cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    c, ctx = (CFG8, CTX8) if big else (CFG, CTX)
    ref = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                         c["vocab_size"], c["max_seq"])
    try:
        ref.synthesize(SEED)
        ref.fill_kv(ctx, SEED)
        toks_ref, logits_ref = _decode(ref, c["vocab_size"], ctx)
    finally:
        ref.close()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, world, port, q, fused, c, ctx, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, off, toks, logits in got:
        assert toks == toks_ref, (rank, toks, toks_ref)
        for step, (lg, lr) in enumerate(zip(logits, logits_ref)):
            sl = lr[off:off + len(lg)]
            assert np.linalg.norm(lg - sl) / np.linalg.norm(sl) <= 1e-3, (rank, step)
