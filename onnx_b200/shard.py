"""Batch sharding across GPUs: one full graph replica per GPU, no collective
on the data path.

Every op of the encoder is independent across batch rows, so a batch is
split into contiguous row slices (rank r gets rows [r*ceil(B/W), ...)), each
rank runs its slice through its own replica, and the host concatenates the
per-rank outputs in rank order.  torch.distributed is used only on the host
(gather of the finished outputs) -- never inside the forward pass.
"""
from __future__ import annotations

import numpy as np


def shard_bounds(batch: int, world: int, rank: int):
    per = -(-batch // world)
    lo = min(rank * per, batch)
    return lo, min(lo + per, batch)


def shard_inputs(inputs: dict, world: int, rank: int) -> dict:
    """Rows of every [B, ...] input that rank `rank` of `world` processes."""
    b = next(iter(inputs.values())).shape[0]
    lo, hi = shard_bounds(b, world, rank)
    return {k: np.ascontiguousarray(v[lo:hi]) for k, v in inputs.items()}


def gather_outputs(local: dict, group=None, batch: int | None = None) -> dict:
    """Concatenate each rank's host outputs in rank order (host-side gather).

    With ``batch`` (the global row count) every output is moved as one
    tensor all_gather of the ceil(batch / world) rows each rank may hold --
    no pickling; without it, as Python objects."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if batch is None:
        parts = [None] * world
        dist.all_gather_object(parts, local, group=group)
        return {k: np.concatenate([p[k] for p in parts], axis=0) for k in local}
    per = -(-batch // world)
    out = {}
    for k in sorted(local):
        a = np.ascontiguousarray(local[k])
        buf = np.zeros((per,) + a.shape[1:], a.dtype)
        buf[:a.shape[0]] = a
        t = torch.from_numpy(buf)
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        out[k] = np.concatenate([parts[r].numpy()[:shard_bounds(batch, world, r)[1] - shard_bounds(batch, world, r)[0]]
                                 for r in range(world)], axis=0)
    return out


def run_sharded(execute, inputs: dict, group=None) -> dict:
    """Run `execute(inputs_slice) -> dict` on this rank's slice and return the
    full-batch outputs on every rank."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    batch = next(iter(inputs.values())).shape[0]
    return gather_outputs(execute(shard_inputs(inputs, world, rank)), group, batch)
