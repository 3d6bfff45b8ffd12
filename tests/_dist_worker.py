"""Worker body of the multi-process sharding tests (spawned, one process per rank).

Every rank builds the same seeded full inputs, takes its shard, runs the
sharded scan forward and backward and saves what it holds for the parent
test to compare with the unsharded scan.
"""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

HERE = Path(__file__).resolve().parent
for p in (HERE, HERE.parent / "mamba-metal-scan_b200", HERE.parent):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from _inputs import inputs  # noqa: E402
from mamba_metal.sharded import (allreduce_aneg_grad, batch_shard, channel_shard,  # noqa: E402
                                 selective_scan_channel_sharded)
from mamba_metal import selective_scan  # noqa: E402


def run(rank: int, world: int, port: int, mode: str, shape, impl: str, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    backend = "nccl" if impl != "torch" else "gloo"
    dev = torch.device("cuda", rank) if backend == "nccl" else torch.device("cpu")
    if backend == "nccl":
        torch.cuda.set_device(dev)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dtype = torch.float64 if impl == "torch" else torch.float32
        bt, t_len, d, n = shape
        x, dt, aneg, b_in, c_in, dy = (t.to(dev) for t in
                                       inputs(bt, t_len, d, n, dist="c0", seed=404, dtype=dtype))
        if mode == "channel":
            sl = channel_shard(d, world, rank)
            leaves = [t.clone().requires_grad_(True) for t in
                      (x[:, :, sl], dt[:, :, sl], aneg[sl], b_in, c_in)]
            y = selective_scan_channel_sharded(*leaves, impl=impl)
            y.backward(dy[:, :, sl])
        else:
            sl = batch_shard(bt, world, rank)
            leaves = [t.clone().requires_grad_(True) for t in
                      (x[sl], dt[sl], aneg, b_in[sl], c_in[sl])]
            y = selective_scan(*leaves, impl=impl)
            y.backward(dy[sl])
            allreduce_aneg_grad(leaves[2])
        torch.save({"slice": (sl.start, sl.stop), "y": y.detach().cpu(),
                    "grads": [t.grad.detach().cpu() for t in leaves]},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()
