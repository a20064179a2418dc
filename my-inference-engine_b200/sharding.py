"""Row sharding of a projection across the GPUs of one node.

The vocabulary projection (src/qwen2_architecture.cpp:1504-1523) is split by
rows: rank r owns rows [r * slot, min(N, (r + 1) * slot)) with
slot = ceil(N / world).  Each rank computes its slice and its argmax key; the
keys combine with an unsigned maximum (largest logit, lowest index on ties,
src/sampler.cpp:29-31) and the slices concatenate in rank order.

``ExchangeGroup`` sets up the peer-memory exchange used by
``Weight.matvec_argmax_exchange``: every rank allocates one exchange buffer,
the 64-byte IPC handles are swapped through a ``torch.distributed`` group
(any backend), and every rank maps its peers' buffers.
"""
from __future__ import annotations

KEY_NONFINITE = 0xFFFFFFFFFFFFFFFF


def shard_rows(n_rows: int, world: int, rank: int):
    """(row_begin, row_end, slot_rows) of `rank`; the last slots may be short."""
    if world < 1 or not 0 <= rank < world or n_rows < 1:
        raise ValueError("bad shard request")
    slot = -(-n_rows // world)
    begin = min(n_rows, rank * slot)
    end = min(n_rows, (rank + 1) * slot)
    return begin, end, slot


def combine_keys(keys) -> int:
    """Global argmax key from per-shard keys (unsigned 64-bit maximum)."""
    out = 0
    for k in keys:
        k = int(k) & 0xFFFFFFFFFFFFFFFF
        if k > out:
            out = k
    return out


def gathered_rows(n_rows: int, world: int):
    """Positions of the N real rows inside the rank-major gathered buffer of
    world * slot entries (slot padding of the last ranks is skipped)."""
    slot = -(-n_rows // world)
    out = []
    for r in range(world):
        b, e, _ = shard_rows(n_rows, world, r)
        out.append((r * slot, r * slot + (e - b)))
    return out


class ExchangeGroup:
    """One rank's view of the exchange buffers of every rank.

    ``ipc`` provides ``exchange_bytes(world, slot)``, ``ipc_alloc(n)`` ->
    (ptr, handle), ``ipc_open(handle)`` -> ptr, ``ipc_close(ptr)`` and
    ``ipc_free(ptr)`` (the library module by default).
    """

    def __init__(self, ipc, rank: int, world: int, slot_rows: int, group=None):
        import torch.distributed as dist

        self.ipc, self.rank, self.world, self.slot_rows = ipc, rank, world, slot_rows
        nbytes = ipc.exchange_bytes(world, slot_rows)
        self.own, handle = ipc.ipc_alloc(nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        if handles[rank] != handle:
            raise RuntimeError("exchange handles arrived out of rank order")
        self.buffers = []
        self.opened = []
        for r, h in enumerate(handles):
            if r == rank:
                self.buffers.append(self.own)
            else:
                ptr = ipc.ipc_open(h)
                self.opened.append(ptr)
                self.buffers.append(ptr)
        self.epoch = 0

    def next_epoch(self, steps: int = 1) -> int:
        """Advance the host's count of exchange calls (the device keeps its own
        counter); returns the epoch of the latest call, which locates its
        gathered logits (qmv_exchange_logits)."""
        self.epoch += steps
        return self.epoch

    def close(self):
        for ptr in self.opened:
            self.ipc.ipc_close(ptr)
        self.opened = []
        if self.own is not None:
            self.ipc.ipc_free(self.own)
            self.own = None
