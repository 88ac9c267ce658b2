"""Host side of the tensor-parallel setup, on CPU: two gloo ranks exchange
their IPC handles through DecodeModel.exchange_handles and each opens the
handles of every rank, in rank order."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _StubModel:
    """Stands in for DecodeModel's handle plumbing (no GPU)."""

    def __init__(self, rank, world):
        self.tp_rank, self.tp_world = rank, world
        self.opened = None

    def comm_handle(self):
        return bytes([self.tp_rank + 1]) * 64

    def comm_open(self, handles):
        self.opened = list(handles)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import guanaco_b200 as gb
        m = _StubModel(rank, world)
        gb.DecodeModel.exchange_handles(m, dist)
        q.put((rank, m.opened))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_handles_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([r + 1]) * 64 for r in range(world)]
    for r in range(world):
        assert got[r] == want
