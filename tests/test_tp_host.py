"""CPU: the tensor-parallel sharding rule and the handle exchange (gloo,
2 ranks), without a GPU."""
import multiprocessing as mp
import os
import socket

import pytest

from blocktensor_b200 import tp


def test_shard_covers_the_model_once():
    for world in (1, 2, 4, 8):
        shards = [tp.shard(32000, 4096, 11008, 32, 32, 128, r, world) for r in range(world)]
        assert sum(s.heads for s in shards) == 32
        assert sum(s.hidden for s in shards) == 11008
        assert sum(s.vocab for s in shards) == 32000
        assert [s.vocab0 for s in shards] == sorted(s.vocab0 for s in shards)
        assert all(s.q_rows % 32 == 0 and s.hidden % 32 == 0 for s in shards)
        # o/down column slices tile the input exactly
        assert [s.o_cols0 for s in shards] == [r * 4096 // world for r in range(world)]
        assert [s.down_cols0 for s in shards] == [r * 11008 // world for r in range(world)]


def test_shard_refusals():
    with pytest.raises(ValueError):
        tp.shard(32000, 4096, 11008, 32, 32, 128, 0, 16)      # above 8 GPUs
    with pytest.raises(ValueError):
        tp.shard(32000, 288, 768, 6, 6, 48, 0, 4)             # 6 heads over 4 GPUs
    with pytest.raises(ValueError):
        tp.shard(32000, 288, 768, 6, 6, 48, 0, 2)             # 3 heads of 48: rows not whole 32-blocks
    s = tp.shard(128256, 8192, 28672, 64, 8, 128, 7, 8)        # 70B shape: one KV head per GPU
    assert (s.kv_heads, s.heads, s.hidden, s.vocab) == (1, 8, 3584, 16032)


class _FakeEngine:
    def __init__(self, rank, world):
        self.tp_rank, self.tp_world = rank, world
        self.connected = None

    def tp_handle(self):
        return bytes([self.tp_rank + 1]) * 64

    def tp_connect(self, handles):
        self.connected = list(handles)


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    e = _FakeEngine(rank, world)
    tp.connect(e)
    q.put((rank, e.connected))
    dist.destroy_process_group()


def test_connect_gathers_handles_in_rank_order():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([1]) * 64, bytes([2]) * 64]
    assert got == {0: want, 1: want}
