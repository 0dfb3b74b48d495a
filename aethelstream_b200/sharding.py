"""Multi-GPU plumbing for the per-layer optimizer step (one process per GPU).

Layers and their weight matrices are independent, so layer ``li`` is owned by
rank ``li % world_size`` and every rank keeps the NF4 weights, projectors and
INT8 state of its own layers only.  The path has exactly two exchanges:

1. the exact global-norm clip needs the sum of all ranks' low-rank squared
   norms (doublepass/src/hook.rs:149-186): one f64 all-reduce per step;
2. a refreshed projector is broadcast from its owner (only to ranks that hold
   a replica; with exclusive sharding it is still timed).

Both go through ``torch.distributed`` (NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def layer_owner(layer_idx: int, world_size: int) -> int:
    """Round-robin assignment of layers to ranks."""
    return layer_idx % world_size


def owned_layers(n_layers: int, rank: int, world_size: int) -> list[int]:
    return [li for li in range(n_layers) if layer_owner(li, world_size) == rank]


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
