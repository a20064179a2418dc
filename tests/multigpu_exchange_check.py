"""Per-rank check of the fused row-sharded projection with its peer-memory
exchange; run under torchrun with one process per GPU (2..8 GPUs).  Exits 0
when, for three steps in a row, every rank's gathered logits are within the
parity bound of the oracle and every rank holds the oracle's greedy token."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import (PKG_DIR, _load, load_oracle_binding, load_package,  # noqa: E402
                      load_workloads, tolerance_ok)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    qmv = load_package()
    qmv.load_library()
    qmv.set_device(local)
    sh = _load("qmv_sharding", os.path.join(PKG_DIR, "sharding.py"))
    wl = load_workloads()
    oracle = load_oracle_binding().Oracle()
    rows, cols = 40001, 3584
    b, e, slot = sh.shard_rows(rows, world, rank)
    blocks = wl.make_blocks(14, rows, cols, seed=6)
    w = qmv.Weight(14, blocks, rows, cols, row_begin=b, row_end=e)
    group = sh.ExchangeGroup(qmv, rank, world, slot)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    host = np.empty(world * slot, np.float32)
    failures = []
    for step in range(3):
        x = wl.make_activations(cols, seed=10 + step)
        xd = torch.from_numpy(x).cuda()
        epoch = group.next_epoch()
        w.matvec_argmax_exchange(xd.data_ptr(), rank, world, group.buffers, slot, key.data_ptr(),
                                 ws.data_ptr())
        torch.cuda.synchronize()
        qmv.memcpy(host, qmv.exchange_logits(group.own, world, slot, epoch), host.nbytes)
        logits = np.concatenate([host[s0:s1] for s0, s1 in sh.gathered_rows(rows, world)])
        y_ref = oracle.matvec(14, blocks, rows, cols, x, threads=8)
        s = oracle.row_abs_dot(14, blocks, rows, cols, x)
        bad = tolerance_ok(logits, y_ref, s)[0]
        ok, want = oracle.argmax(y_ref)
        tok = qmv.key_to_token(int(key.cpu().numpy().view(np.uint64)[0]))
        if bad.size or not ok or tok != want:
            failures.append((step, int(bad.size), tok, want))
    status = qmv.device_status()
    dist.barrier()
    group.close()
    w.free()
    dist.destroy_process_group()
    if failures or status:
        print(f"rank {rank}: failures {failures} status {status}", flush=True)
        sys.exit(1)
    print(f"rank {rank}: ok", flush=True)


if __name__ == "__main__":
    main()
