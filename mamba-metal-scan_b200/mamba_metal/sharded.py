"""The scan split across the GPUs of one node, one process per GPU.

The recurrence is independent per (batch row, channel), so it shards without
any exchange inside the scan:

* Batch sharding: rank r scans its own rows (`batch_shard`). Nothing is
  exchanged; y, dx, ddt, dB, dC of a row live on the rank that owns it. dAneg
  is a per-rank partial sum over that rank's rows: `allreduce_aneg_grad` sums
  it (D*N floats) when the ranks train one shared Aneg, as data parallelism
  does.
* Channel (d_inner) sharding: rank r owns channels `channel_shard(D, P, r)`,
  i.e. its slice of x, dt and Aneg, while B and C (B, T, N) are replicated.
  y, dx, ddt and dAneg stay local. dB and dC are sums over all channels, so
  every rank holds a partial; `selective_scan_channel_sharded` sums the
  packed [dB | dC] buffer (2*B*T*N floats) with one all-reduce over the
  process group (NCCL over NVLink on GPUs, gloo on CPU).

The scan itself runs through `mamba_metal.selective_scan` with the caller's
`impl`, so on CUDA tensors it is the native kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from mamba_metal.scan import SSM_CHUNK, selective_scan


def _split(total: int, parts: int, index: int, multiple: int = 1) -> slice:
    """Contiguous near-equal split of range(total) into `parts`; piece `index`.

    Piece sizes are multiples of `multiple` where the total allows it (the
    remainder goes to the last piece), so every shard keeps 16-byte rows.
    """
    if parts < 1 or not 0 <= index < parts:
        raise ValueError(f"bad shard index {index} of {parts}")
    units = total // multiple
    base, extra = divmod(units, parts)
    start = (index * base + min(index, extra)) * multiple
    stop = start + (base + (1 if index < extra else 0)) * multiple
    if index == parts - 1:
        stop = total
    return slice(start, stop)


def batch_shard(batch: int, world: int, rank: int) -> slice:
    """Rows of the batch that rank `rank` of `world` scans."""
    return _split(batch, world, rank)


def channel_shard(d_inner: int, world: int, rank: int) -> slice:
    """Channels (d_inner) that rank `rank` of `world` owns; multiples of 4 where possible."""
    return _split(d_inner, world, rank, multiple=4 if d_inner >= 4 * world else 1)


class _SumGradAcrossRanks(torch.autograd.Function):
    """Identity forward; all-reduce (sum) of the gradient in backward.

    Marks the point where a replicated input (here the packed [B | C]) enters
    per-rank computation: each rank's gradient is a partial sum over its own
    channels, and the full gradient is their sum.
    """

    @staticmethod
    def forward(ctx, t, group):
        ctx.group = group
        return t.view_as(t)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=ctx.group)
        return grad, None


def selective_scan_channel_sharded(x: torch.Tensor, dt: torch.Tensor, aneg: torch.Tensor,
                                   b_in: torch.Tensor, c_in: torch.Tensor,
                                   group=None, impl: str = "auto", chunk: int = SSM_CHUNK,
                                   return_state: bool = False):
    """The scan over this rank's channels, with dB/dC summed over the group.

    x, dt (B, T, D_local) and Aneg (D_local, N) are this rank's channel slice
    (`channel_shard`); B, C (B, T, N) are the same on every rank. Returns this
    rank's y (B, T, D_local) (and its (B, D_local, N) state with
    return_state). Backward gives local dx, ddt, dAneg and the full dB, dC,
    identical on every rank, from one all-reduce of the packed [dB | dC].
    """
    bc = torch.stack((b_in, c_in))                       # (2, B, T, N), replicated
    if torch.is_grad_enabled() and bc.requires_grad and dist.is_initialized():
        bc = _SumGradAcrossRanks.apply(bc, group)
    out = selective_scan(x, dt, aneg, bc[0], bc[1], impl=impl, chunk=chunk,
                         return_state=return_state)
    if out is None:
        raise RuntimeError(f"scan_impl={impl!r} declined tensors on {x.device}; use 'torch' "
                           "on the CPU or CUDA tensors")
    return out


def allreduce_aneg_grad(aneg: torch.Tensor, group=None) -> None:
    """Sum Aneg's gradient over the ranks of a batch-sharded (data-parallel) scan."""
    if aneg.grad is not None and dist.is_initialized():
        dist.all_reduce(aneg.grad, op=dist.ReduceOp.SUM, group=group)
