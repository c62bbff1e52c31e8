"""Data-parallel sharding of the attention path over ranks (one process per GPU).

The units of this path are independent: a decode step attends each sequence to its own
KV cache, a prefill attends each sequence to itself.  So a batch spread over N GPUs needs
no exchange while it is computed: every rank takes an equal number of sequences, chosen
so that the ranks' costs (visible keys) balance, computes them with the single-GPU entry
points, and only a caller that wants the whole batch's output in one place gathers it
afterwards (one all-gather of equal-size shards).  The reference runs on one GPU and has
no counterpart of this module.
"""
from __future__ import annotations

import numpy as np


def plan_shards(unit_cost, world: int) -> list[np.ndarray]:
    """Ascending unit indices per rank: equal counts, costs balanced (longest first onto
    the least-loaded rank that still has room) by the library's b2a_partition_units.
    len(unit_cost) must be a multiple of `world`; every rank computing the plan from the
    same costs gets the same plan."""
    from . import partition_units
    owner = partition_units(np.asarray(unit_cost, dtype=np.int64), world)
    return [np.flatnonzero(owner == r) for r in range(world)]


def _device_of(group):
    import torch
    import torch.distributed as dist
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")


class Reassembly:
    """Output reassembly for one plan, set up once: one all-gather of the equal shards into a
    single buffer (rank-major), then one index copy back into unit order on the receiving
    device.  The unit-order index lives on the device, so a call issues no host-device copy
    and no synchronisation."""

    def __init__(self, plan: list[np.ndarray], device):
        import torch
        counts = {len(p) for p in plan}
        if len(counts) != 1:
            raise ValueError("gather_shards needs equal shard sizes (use plan_shards)")
        self.world, self.per = len(plan), counts.pop()
        # gathered row i holds unit order[i]
        self.order = torch.as_tensor(np.concatenate(plan), dtype=torch.long, device=device)

    def __call__(self, local, group=None):
        import torch
        import torch.distributed as dist
        if local.shape[0] != self.per:
            raise ValueError("local results do not match this rank's shard size")
        buf = local.new_empty((self.world * self.per,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
        out = torch.empty_like(buf)
        out.index_copy_(0, self.order, buf)
        return out


def gather_shards(local, plan: list[np.ndarray], group=None):
    """Reassembles per-rank results into global unit order on every rank.

    local: this rank's results, [len(plan[rank]), ...] in the order of plan[rank].
    Returns [n_units, ...].  Shards are equal in size (plan_shards), so one all-gather
    moves them; the scatter back into unit order happens on the receiving device.  A
    caller that reassembles every step builds a Reassembly once instead."""
    return Reassembly(plan, local.device)(local, group)


def max_over_ranks(values, group=None) -> list[float]:
    """Elementwise maximum over ranks of per-rank numbers (device-timed durations): the
    whole job is as slow as its slowest rank."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return [float(v) for v in values]  # one process: nothing to reduce
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=_device_of(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t.cpu()]
