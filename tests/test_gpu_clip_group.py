"""The global clip over a group of GPUs through peer memory.

The squared-norm launch of aeth_galore_step writes this GPU's sum into a slot
on every group member and reads theirs (bounded wait).  On one GPU the group
is emulated with a second slot buffer standing for the peer: the test writes
the "peer's" sum into this GPU's slots before each step and reads back what
the kernel stored for the peer.  The result must equal, bit for bit, the step
whose squared-norm hook adds the same value (the NCCL path of
doublepass/src/hook.rs:149-186).  A peer that never writes makes the wait
give up: clip 0 and the peer-timeout bit in the device error word, with the
context still usable.  With two GPUs, two processes form a real group and
must match two processes that exchange the sums through a host hook.
"""
import os
import socket
import struct

import numpy as np
import pytest
import torch

from tests._gpu import host

pytestmark = pytest.mark.gpu

SPECS = [(0, "d_wq", 256, 512, 64), (0, "d_wk", 512, 256, 64), (0, "d_wg", 256, 256, 32)]


def _opt(**kw):
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig
    cfg = GaLoreConfig(mode="b200", layer_ranks=LayerRankConfig(), svd_refresh=False, max_grad_norm=0.01, **kw)
    return GaLoreOptimizer(cfg, SPECS, device=torch.cuda.current_device())


def _dev(a):
    """To the current device (the two-GPU workers run on cuda:1 too)."""
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.device("cuda", torch.cuda.current_device()))


def _inputs(seed):
    from aethelstream_b200 import nf4_quantize
    rng = np.random.default_rng(seed)
    gs = [[_dev((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)).to(torch.bfloat16)
           for _, _, m, n, _ in SPECS] for _ in range(3)]
    ws = [nf4_quantize(_dev((rng.standard_normal((m, n)) * 0.02).astype(np.float32))) for _, _, m, n, _ in SPECS]
    return gs, ws


def _slot_view(addr, world):
    """int64 view of a slot buffer: [parity][world] x {f64 sum bits, epoch}."""
    class _H:
        __cuda_array_interface__ = {"shape": (2 * world * 2,), "typestr": "<i8", "data": (addr, False),
                                    "version": 2, "strides": None}
    return torch.as_tensor(_H(), device=torch.device("cuda", torch.cuda.current_device()))


def _f64_bits(x):
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def _bits_f64(b):
    return struct.unpack("<d", struct.pack("<Q", int(b)))[0]


def _state(opt, ws):
    out = [host(w.packed) for w in ws] + [host(w.absmax) for w in ws]
    for li, nm, *_ in SPECS:
        out += [host(x) for x in opt.get_state(li, nm)]
    return out


def _keys():
    return [(li, nm) for li, nm, *_ in SPECS]


def test_emulated_peer_equals_hook():
    from aethelstream_b200 import _lib
    peer_sums = [3.0e-4, 1.25e-4, 7.5e-5]
    # the hook path: the host adds the peer's sum after the local one (rank order)
    gs, ws = _inputs(5)
    opt = _opt()
    local_seen = []

    def hook(sq):
        vals = sq.cpu().tolist()
        t = 0.0
        for v in vals:
            t += v
        local_seen.append(t)
        sq.zero_()
        sq[0] = t + peer_sums[len(local_seen) - 1]
    clips_hook = [float(host(opt.step_layer(_keys(), g, ws, sq_hook=hook))[0]) for g in gs]
    ref = _state(opt, ws)
    opt.close()

    # the group path: rank 0 of 2, the peer's sums prefilled into this GPU's slots
    gs, ws = _inputs(5)
    opt = _opt()
    opt.clip_handle(2)
    own = opt.clip_slots()
    peer_buf = torch.zeros(2 * 2 * 2, dtype=torch.int64, device=torch.device("cuda", torch.cuda.current_device()))
    opt.set_clip_group_ptrs(0, [own, peer_buf.data_ptr()], timeout_s=2.0)
    own_v = _slot_view(own, 2)
    clips_grp = []
    for e, g in enumerate(gs, start=1):
        par = e & 1
        entry = torch.tensor([_f64_bits(peer_sums[e - 1]), e], dtype=torch.int64).to(own_v.device)
        own_v[(par * 2 + 1) * 2:(par * 2 + 1) * 2 + 2].copy_(entry)
        clips_grp.append(float(host(opt.step_layer(_keys(), g, ws))[0]))
        written = host(peer_buf).view(np.uint64)
        # this GPU's sum, stored into the peer's slot [parity][rank 0] with the epoch after it
        assert int(written[(par * 2 + 0) * 2 + 1]) == e
        assert _bits_f64(written[(par * 2 + 0) * 2]) == local_seen[e - 1]
    assert _lib.device_error_bits(torch.cuda.current_device()) == 0
    got = _state(opt, ws)
    opt.close()
    assert clips_grp == clips_hook and all(c < 1.0 for c in clips_grp)
    for x, y in zip(got, ref):
        assert np.array_equal(x, y)


def test_missing_peer_times_out():
    from aethelstream_b200 import _lib
    gs, ws = _inputs(9)
    opt = _opt()
    opt.clip_handle(2)
    peer_buf = torch.zeros(8, dtype=torch.int64, device=torch.device("cuda", torch.cuda.current_device()))
    d = torch.cuda.current_device()
    _lib.device_error_bits(d)  # start clean
    opt.set_clip_group_ptrs(0, [opt.clip_slots(), peer_buf.data_ptr()], timeout_s=0.05)
    clip = float(host(opt.step_layer(_keys(), gs[0], ws))[0])
    bits = _lib.device_error_bits(d)
    assert clip == 0.0
    assert bits & _lib.DEVERR_TIMEOUT_PEER
    # the context stays usable: leave the group and step locally
    opt.set_clip_group(0, 1, [])
    clip = float(host(opt.step_layer(_keys(), gs[1], ws))[0])
    assert 0.0 < clip < 1.0
    assert _lib.device_error_bits(d) == 0
    opt.close()


def test_group_requires_b200_mode_and_matching_slots():
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig, _lib
    opt = _opt()
    with pytest.raises(_lib.AethError):
        opt.set_clip_group_ptrs(0, [1 << 40, 1 << 41])  # no slots allocated yet
    opt.clip_handle(2)
    with pytest.raises(_lib.AethError):
        opt.set_clip_group_ptrs(0, [opt.clip_slots() + 64, opt.clip_slots()])  # own slots not at `rank`
    opt.close()
    ref = GaLoreOptimizer(GaLoreConfig(mode="ref", layer_ranks=LayerRankConfig()), [(0, "d_wq", 64, 64)], device=0)
    with pytest.raises(_lib.AethError):
        ref.set_clip_group(0, 2, [b"\0" * 64, b"\0" * 64])
    ref.close()


# --------------------------------------------------------------------------- two GPUs
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_gpu_worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from aethelstream_b200 import _lib
        from aethelstream_b200.sharding import setup_clip_group
        gs, ws = _inputs(100 + rank)
        opt = _opt()
        if mode == "group":
            assert setup_clip_group(opt, timeout_s=5.0)
            clips = [float(host(opt.step_layer(_keys(), g, ws))[0]) for g in gs]
        elif mode == "hook":
            def hook(sq):
                t = 0.0
                for v in sq.cpu().tolist():
                    t += v
                every = [None] * world
                dist.all_gather_object(every, t)
                total = 0.0
                for v in every:
                    total += v
                sq.zero_()
                sq[0] = total
            clips = [float(host(opt.step_layer(_keys(), g, ws, sq_hook=hook))[0]) for g in gs]
        else:  # "leave": rank 1 joins but skips the step
            assert setup_clip_group(opt, timeout_s=0.1)
            clips = []
            if rank == 0:
                clips = [float(host(opt.step_layer(_keys(), gs[0], ws))[0])]
            dist.barrier()
        bits = _lib.device_error_bits(rank)
        opt.set_clip_group(0, 1, [])
        q.put((mode, rank, clips, bits, [x.tobytes() for x in _state(opt, ws)]))
        dist.barrier()
        opt.close()
    finally:
        dist.destroy_process_group()


def _run_two(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=240) for _ in range(2)), key=lambda x: x[1])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_group_equals_host_exchange():
    grp = _run_two("group")
    hk = _run_two("hook")
    for (_, r, c_g, b_g, s_g), (_, _, c_h, b_h, s_h) in zip(grp, hk):
        assert b_g == 0 and b_h == 0
        assert c_g == c_h and all(c < 1.0 for c in c_g), (r, c_g, c_h)
        assert s_g == s_h
    assert grp[0][2] == grp[1][2]  # every rank has the same clip bits


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_rank_that_skips_a_step():
    from aethelstream_b200 import _lib
    res = _run_two("leave")
    (_, _, clips0, bits0, _), (_, _, clips1, bits1, _) = res
    assert clips0 == [0.0] and bits0 & _lib.DEVERR_TIMEOUT_PEER
    assert clips1 == [] and bits1 == 0
