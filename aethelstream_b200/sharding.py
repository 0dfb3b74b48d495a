"""Multi-GPU plumbing for the per-layer optimizer step (one process per GPU).

Layers and their weight matrices are independent, so layer ``li`` is owned by
rank ``li % world_size`` and every rank keeps the NF4 weights, projectors and
INT8 state of its own layers only.  The path has exactly two exchanges:

1. the exact global-norm clip needs the sum of all ranks' low-rank squared
   norms (doublepass/src/hook.rs:149-186).  On B200s the squared-norm kernel
   exchanges it itself: every rank stores its sum into a slot on each peer
   GPU over NVLink and reads theirs (``setup_clip_group``), inside the launch
   that computes the norms.  ``allreduce_sqnorm_hook`` is the alternative
   through a ``torch.distributed`` all-reduce (NCCL, or gloo on CPU);
2. a refreshed projector is broadcast from its owner (only to ranks that hold
   a replica; with exclusive sharding it is still timed).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def layer_owner(layer_idx: int, world_size: int) -> int:
    """Round-robin assignment of layers to ranks."""
    return layer_idx % world_size


def owned_layers(n_layers: int, rank: int, world_size: int) -> list[int]:
    return [li for li in range(n_layers) if layer_owner(li, world_size) == rank]


def setup_clip_group(optimizer, group=None, timeout_s: float = 2.0) -> bool:
    """Joins every rank's optimizer into one peer-memory clip group: each
    rank allocates its slots and publishes their IPC handle, the handles are
    gathered in rank order, each rank opens its peers' slots, and the ranks
    agree on the outcome (the agreement doubles as the barrier the group
    needs before its first step).  Returns True when every rank joined;
    otherwise every rank leaves the group and the caller exchanges the norms
    another way (``allreduce_sqnorm_hook``).  Every rank takes the same
    collective steps on either outcome."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if world == 1:
        optimizer.set_clip_group(0, 1, [])
        return True
    try:
        handle, err = optimizer.clip_handle(world), ""
    except Exception as e:  # noqa: BLE001 - reported to every rank below
        handle, err = b"", repr(e)
    handles: list = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    if not err:
        try:
            if any(not h for h in handles):
                raise RuntimeError("a rank has no clip handle")
            optimizer.set_clip_group(rank, world, handles, timeout_s)
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            err = repr(e)
    outcomes: list = [None] * world
    dist.all_gather_object(outcomes, err, group=group)
    if any(outcomes):
        if not err:
            optimizer.set_clip_group(0, 1, [])
        return False
    return True


def allreduce_sqnorm_hook(group=None):
    """A ``GaLoreOptimizer.step_layer`` sq_hook: replaces the local
    per-parameter squared norms by [global sum, 0, 0, ...] so that the device
    clip kernel, which sums the array, sees the sum over all ranks."""
    def hook(sq: torch.Tensor) -> None:
        total = sq.sum().reshape(1)
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
        sq.zero_()
        sq[:1].copy_(total)
    return hook


def global_clip_coeff(local_sqnorms, max_grad_norm: float, group=None, device=None) -> tuple[float, float]:
    """Host-side global clip over all ranks (hook.rs:184-187).  Returns
    (global_grad_norm, clip_coeff)."""
    import numpy as np
    t = torch.tensor([float(sum(local_sqnorms))], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    gnorm = float(t.item()) ** 0.5
    max_norm = float(np.float32(max_grad_norm))
    clip = min(float(np.float32(max_norm / (gnorm + 1e-6))), 1.0)
    return gnorm, clip


def broadcast_projector(proj: torch.Tensor, owner: int, group=None) -> torch.Tensor:
    """Broadcast a refreshed projector from its owning rank (in place)."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.broadcast(proj, src=owner, group=group)
    return proj
