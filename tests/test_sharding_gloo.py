"""Multi-rank host logic on CPU (gloo, world_size 2): round-robin layer
ownership, the exact global clip over all ranks' squared norms, the device-
clip hook's all-reduce, and the projector broadcast from its owner."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aethelstream_b200 import sharding
        n_layers = 5
        mine = sharding.owned_layers(n_layers, rank, world)
        # synthetic per-layer squared norms, the same table on every rank
        table = [float(1.5 * (li + 1)) for li in range(n_layers)]
        gnorm, clip = sharding.global_clip_coeff([table[li] for li in mine], 1.0)
        # device-clip hook semantics on CPU tensors
        sq = torch.tensor([table[li] for li in mine] + [0.0], dtype=torch.float64)
        sharding.allreduce_sqnorm_hook()(sq)
        proj = torch.full((4, 3), float(rank), dtype=torch.float32)
        sharding.broadcast_projector(proj, owner=sharding.layer_owner(3, world))
        q.put((rank, mine, gnorm, clip, sq.tolist(), proj[0, 0].item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_clip_and_broadcast():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    table = [1.5 * (li + 1) for li in range(5)]
    total = sum(table)
    expect_clip = min(float(np.float32(1.0 / (total ** 0.5 + 1e-6))), 1.0)
    owned = sorted(li for _, mine, *_ in res for li in mine)
    assert owned == list(range(5))
    assert res[0][1] == [0, 2, 4] and res[1][1] == [1, 3]
    for rank, mine, gnorm, clip, sq, b in res:
        assert abs(gnorm - total ** 0.5) < 1e-12
        assert clip == expect_clip
        assert abs(sq[0] - total) < 1e-12 and all(v == 0.0 for v in sq[1:])
        assert b == 1.0  # layer 3 belongs to rank 1


class _FakeGroupOptimizer:
    """Records the clip-group calls of sharding.setup_clip_group (host logic only)."""

    def __init__(self, rank, fail_join):
        self.rank, self.fail_join, self.calls = rank, fail_join, []

    def clip_handle(self, world):
        self.calls.append(("handle", world))
        return bytes([self.rank + 1]) * 64

    def set_clip_group(self, rank, world, handles, timeout_s=2.0):
        self.calls.append(("join", rank, world, [h[0] for h in handles]))
        if self.fail_join and world > 1:
            raise RuntimeError("cannot open the peer's handle")


def _group_worker(rank, world, port, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aethelstream_b200 import sharding
        opt = _FakeGroupOptimizer(rank, fail_join=(rank == fail_rank))
        ok = sharding.setup_clip_group(opt)
        q.put((rank, ok, opt.calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_setup_clip_group_agrees_on_outcome(fail_rank):
    """Handles are gathered in rank order; if any rank cannot join, every rank
    leaves the group and reports False (same collective steps either way)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_group_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, ok, calls in res:
        assert calls[0] == ("handle", 2)
        assert calls[1] == ("join", rank, 2, [1, 2])  # every rank's handle, in rank order
        assert ok == (fail_rank < 0)
        if fail_rank < 0:
            assert len(calls) == 2
        elif rank != fail_rank:
            assert calls[2] == ("join", 0, 1, [])  # left the group again
