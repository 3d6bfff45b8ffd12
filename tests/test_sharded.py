"""Sharding of the scan across ranks: host logic on CPU ranks (gloo).

Batch sharding needs no exchange; channel (d_inner) sharding needs one
all-reduce of the packed [dB | dC] partials (mamba_metal/sharded.py). Two
gloo ranks run the sharded scan with the PyTorch implementation in float64;
their outputs, stitched together, must equal the unsharded scan. The same
test on two GPUs over NCCL with the CUDA kernels is marked gpu and needs two
devices.
"""
from __future__ import annotations

import socket

import pytest
import torch
import torch.multiprocessing as mp

import _dist_worker
from _inputs import inputs, max_rel
from mamba_metal import selective_scan
from mamba_metal.sharded import batch_shard, channel_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(mode, shape, impl, tmp_path, world=2):
    mp.start_processes(_dist_worker.run, args=(world, _free_port(), mode, shape, impl,
                                               str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    return [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]


def _full(shape, impl, dtype, device="cpu"):
    bt, t_len, d, n = shape
    x, dt, aneg, b_in, c_in, dy = (t.to(device) for t in
                                   inputs(bt, t_len, d, n, dist="c0", seed=404, dtype=dtype))
    leaves = [t.clone().requires_grad_(True) for t in (x, dt, aneg, b_in, c_in)]
    y = selective_scan(*leaves, impl=impl)
    y.backward(dy)
    return y.detach().cpu(), [t.grad.detach().cpu() for t in leaves]


def test_shard_splits_cover_the_range_once():
    for total in (1, 3, 8, 10, 17, 2048, 8192):
        for world in (1, 2, 3, 4, 8):
            if world > total:
                continue
            for fn in (batch_shard, channel_shard):
                pieces = [fn(total, world, r) for r in range(world)]
                assert pieces[0].start == 0 and pieces[-1].stop == total
                assert all(a.stop == b.start for a, b in zip(pieces, pieces[1:]))
                assert all(p.stop > p.start for p in pieces)
    # channel shards keep 16-byte rows when D allows it
    assert [channel_shard(8192, 8, r).stop - channel_shard(8192, 8, r).start
            for r in range(8)] == [1024] * 8
    assert all((channel_shard(2052, 8, r).start % 4) == 0 for r in range(8))
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


def _check(results, shape, mode, impl, dtype, tol, device="cpu"):
    y_full, g_full = _full(shape, impl, dtype, device)
    for r in results:
        sl = slice(*r["slice"])
        gx, gdt, ganeg, gb, gc = r["grads"]
        if mode == "channel":
            assert max_rel(r["y"], y_full[:, :, sl]) <= tol
            assert max_rel(gx, g_full[0][:, :, sl]) <= tol
            assert max_rel(gdt, g_full[1][:, :, sl]) <= tol
            assert max_rel(ganeg, g_full[2][sl]) <= tol
            assert max_rel(gb, g_full[3]) <= tol      # summed over the ranks' channels
            assert max_rel(gc, g_full[4]) <= tol
        else:
            assert max_rel(r["y"], y_full[sl]) <= tol
            assert max_rel(gx, g_full[0][sl]) <= tol
            assert max_rel(gdt, g_full[1][sl]) <= tol
            assert max_rel(ganeg, g_full[2]) <= tol   # summed over the ranks' rows
            assert max_rel(gb, g_full[3][sl]) <= tol
            assert max_rel(gc, g_full[4][sl]) <= tol


@pytest.mark.parametrize("mode,shape", [("channel", (2, 13, 10, 8)), ("channel", (1, 9, 16, 4)),
                                        ("batch", (3, 11, 6, 8))])
def test_two_gloo_ranks_match_the_unsharded_scan(mode, shape, tmp_path):
    results = _launch(mode, shape, "torch", tmp_path)
    _check(results, shape, mode, "torch", torch.float64, 1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("mode,shape", [("channel", (2, 300, 520, 16)), ("batch", (4, 257, 96, 16))])
def test_two_nccl_ranks_match_the_unsharded_scan(mode, shape, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    results = _launch(mode, shape, "cuda", tmp_path)
    _check(results, shape, mode, "cuda", torch.float32, 1e-4, device="cuda")
