"""Host logic of the multi-GPU path on CPU, with world_size-2 gloo ranks.

* row shards cover every row exactly once, in rank order;
* per-shard argmax keys (computed here from the oracle's logits) combined
  across ranks give the oracle's greedy token over the whole vocabulary;
* ExchangeGroup routes IPC handles by rank and opens exactly the peers'
  buffers (the CUDA IPC calls are replaced by a recording fake: no GPU).
"""
import os
import socket
import struct

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import load_oracle_binding, load_workloads, PKG_DIR, _load


def sharding():
    return _load("qmv_sharding", os.path.join(PKG_DIR, "sharding.py"))


def py_key(v: float, index: int) -> int:
    u = struct.unpack("<I", struct.pack("<f", v))[0]
    if (u & 0x7F800000) == 0x7F800000:
        return 0xFFFFFFFFFFFFFFFF
    if (u & 0x7FFFFFFF) == 0:
        u = 0
    o = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (o << 32) | (0xFFFFFFFF - index)


@pytest.mark.parametrize("n,world", [(152064, 8), (152064, 3), (10, 4), (7, 8), (1, 2)])
def test_shards_cover_rows_once(n, world):
    sh = sharding()
    seen = []
    for r in range(world):
        b, e, slot = sh.shard_rows(n, world, r)
        assert 0 <= b <= e <= n and e - b <= slot
        seen.extend(range(b, e))
    assert seen == list(range(n))
    spans = sh.gathered_rows(n, world)
    assert sum(e - b for b, e in spans) == n


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeIpc:
    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.freed = [], [], []

    def exchange_bytes(self, world, slot):
        return 2 * world * slot * 4

    def ipc_alloc(self, n):
        return 1000 + self.rank, bytes([self.rank]) * 64

    def ipc_open(self, handle):
        self.opened.append(handle[0])
        return 2000 + handle[0]

    def ipc_close(self, ptr):
        self.closed.append(ptr)

    def ipc_free(self, ptr):
        self.freed.append(ptr)


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = sharding()
        wl = load_workloads()
        oracle = load_oracle_binding().Oracle()
        rows, cols = 3000, 512
        b, e, slot = sh.shard_rows(rows, world, rank)
        blocks = wl.make_blocks(14, rows, cols, seed=4, row_begin=b, row_end=e)
        x = wl.make_activations(cols, seed=4)
        y = oracle.matvec(14, blocks, e - b, cols, x)
        local_key = max(py_key(float(v), b + i) for i, v in enumerate(y))
        keys = [None] * world
        dist.all_gather_object(keys, local_key)
        token = struct.unpack("<I", struct.pack("<I", 0xFFFFFFFF - (sh.combine_keys(keys) & 0xFFFFFFFF)))[0]
        fake = FakeIpc(rank)
        g = sh.ExchangeGroup(fake, rank, world, slot)
        buffers = list(g.buffers)
        g.close()
        q.put((rank, token, buffers, sorted(fake.opened), sorted(fake.closed), fake.freed))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_combine_and_handle_routing():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, token, buffers, opened, closed, freed = q.get(timeout=120)
        results[rank] = (token, buffers, opened, closed, freed)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    wl = load_workloads()
    oracle = load_oracle_binding().Oracle()
    blocks = wl.make_blocks(14, 3000, 512, seed=4)
    x = wl.make_activations(512, seed=4)
    ok, want = oracle.argmax(oracle.matvec(14, blocks, 3000, 512, x))
    assert ok
    for rank, (token, buffers, opened, closed, freed) in results.items():
        assert token == want
        assert buffers[rank] == 1000 + rank
        peers = [r for r in range(world) if r != rank]
        assert opened == peers
        assert [buffers[r] for r in peers] == [2000 + r for r in peers]
        assert closed == [2000 + r for r in peers] and freed == [1000 + rank]
