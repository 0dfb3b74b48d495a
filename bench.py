"""Benchmark of the per-layer optimizer step (NF4 -> GaLore -> INT8 Adam -> NF4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload ("C2"): one Llama-2-7B decoder block per GPU --
q/k/v/o 4096x4096, gate/up 11008x4096, down 4096x11008 -- NF4 weights
N(0, 0.02), bf16 gradients N(0, 1e-3), GaLore rank 128 on the smaller
dimension with fixed projectors, INT8 blockwise dynamic-map Adam state, 50
consecutive steps by default.  A step is one full optimizer step of the block
through the public API (GaLoreOptimizer.step_layer): projection of all seven
gradients, exact global-norm clip on the device, Adam, back-projection and the
NF4 weight write.  Gradients cycle through a two-deep ring generated on the
device from seeds (step parity, matrix); all weights and state stay resident.
Under torchrun each rank owns one block (weak scaling); the only exchange is
the f64 all-reduce of the squared norms for the global clip.

The reference arm (--impl reference) times the reference's CPU algorithm
(oracle/ port of galore/src/{project,adamw,optimizer}.rs, nf4.rs; the Rust
crate cannot be built here) on all host threads over a bounded row sample of
the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "params updated/s (NF4->GaLore->INT8-Adam step)"
UNIT = "params/s"
CONFIGS = {
    # the bench workload
    "c2": dict(shapes=[("d_wq", 4096, 4096), ("d_wk", 4096, 4096), ("d_wv", 4096, 4096), ("d_wo", 4096, 4096),
                       ("d_wg", 11008, 4096), ("d_wu", 11008, 4096), ("d_wd", 4096, 11008)],
               workload=("C2: one Llama-2-7B block per GPU (q/k/v/o 4096x4096, gate/up 11008x4096, down 4096x11008), "
                         "GaLore r=128 one-sided on the smaller dim, fixed projectors, NF4 weights, bf16 grads, "
                         "INT8 blockwise-2048 dynamic-map Adam, fused NF4 requant")),
    # one 4096x4096 weight (used for small profiling captures)
    "c1": dict(shapes=[("d_wq", 4096, 4096)],
               workload=("C1: one 4096x4096 weight, GaLore r=128, NF4 weight, bf16 grad, "
                         "INT8 blockwise-2048 dynamic-map Adam, fused NF4 requant")),
}
SHAPES = CONFIGS["c2"]["shapes"]
RANK = 128
STATE_BLOCK = 2048
WORKLOAD = CONFIGS["c2"]["workload"]


def algorithmic(shapes=None, r=RANK):
    """Algorithmic bytes and flops per step, split by phase.

    projection phase (K4): read bf16 G (2 B/elem) + projector (2 s r).
    apply phase (K5+K6): NF4 weight read + write (2 x 0.5625 B/elem), INT8 m/v
    read + write (4 r l), block scales (8 r l / 2048), projector (2 s r).
    Flops: 2 r m n per GEMM (projection and back-projection) + ~12 r l (Adam).
    """
    bp = ba = fp = fa = 0
    for _, m, n in (shapes or SHAPES):
        s, l = min(m, n), max(m, n)
        bp += 2 * m * n + 2 * s * r
        ba += 2 * 0.5625 * m * n + 4 * r * l + 8 * r * l / STATE_BLOCK + 2 * s * r
        fp += 2 * r * m * n
        fa += 2 * r * m * n + 12 * r * l
    return {"proj_bytes": bp, "apply_bytes": ba, "proj_flops": fp, "apply_flops": fa}


KERNEL_NAMES = {
    "projection": "proj_grouped_kernel (tcgen05 one-sided projection, TMA reduce-add into R)",
    "sqnorm_clip": "sqnorm_group_kernel (f64 squared norms + global clip)",
    "adam": "b2_adam_group_kernel (INT8 dynamic-map Adam, N in bf16)",
    "apply": "apply_grouped_kernel (tcgen05 back-projection + fused NF4 dequant/update/requant)",
}


def kernel_bytes(shapes=None, r=RANK):
    """Compulsory HBM bytes per launch of each step kernel (one launch each per step).

    projection: read G bf16 (2 B/elem) + projector (2 s r), write R f32 (4 r l).
    sqnorm_clip: read R (4 r l).
    adam: read R + zero R (8 r l), m/v codes read + write (4 r l), N bf16 write (2 r l),
          block scales read + write (16 r l / 2048).
    apply: NF4 weight read + write (2 x 0.5625 B/elem), N bf16 read (2 r l), projector (2 s r).
    """
    out = dict.fromkeys(("projection", "sqnorm_clip", "adam", "apply"), 0.0)
    for _, m, n in (shapes or SHAPES):
        s, l = min(m, n), max(m, n)
        out["projection"] += 2 * m * n + 2 * s * r + 4 * r * l
        out["sqnorm_clip"] += 4 * r * l
        out["adam"] += 14 * r * l + 16 * r * l / STATE_BLOCK
        out["apply"] += 2 * 0.5625 * m * n + 2 * r * l + 2 * s * r
    return out


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summary (if present)."""
    p = os.path.join(ROOT, "profiles", "traffic_c2.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:  # noqa: BLE001
            return {}
    return {}


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed
    region: NVML in a thread every 10 ms (read-only queries), else
    nvidia-smi -lms 200."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = False
        self.thread = None
        self.proc = None

    def _nvml_loop(self, nv, h):
        while not self._stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.samples.append((sm, get(h)))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.01)

    def start(self):
        try:
            import threading

            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self._physical_index())
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001 - no NVML: report no clocks
            self.thread = None

    def _physical_index(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                return int(vis.split(",")[self.idx])
            except (ValueError, IndexError):
                return self.idx
        return self.idx

    def stop(self):
        if self.thread is None:
            return None
        self._stop = True
        self.thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        sm = [s for s, _ in self.samples]
        reasons = sorted({name for _, rs in self.samples for bit, name in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def cpu_baseline(frac, threads, k=1):
    """The reference algorithm (oracle port) on a bounded row sample."""
    from oracle import oracle as O
    O.build()
    samp = O.ReferenceSampler([(m, n) for _, m, n in SHAPES], RANK, frac, threads=threads, seed=1)
    samp.step()  # warm caches
    t0 = time.perf_counter()
    done = 0.0
    for _ in range(k):
        done += samp.step()
    dt = time.perf_counter() - t0
    return done / dt, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    frac = 1.0 / 64
    from oracle import oracle as O
    O.build()
    samp = O.ReferenceSampler([(m, n) for _, m, n in SHAPES], RANK, frac, threads=threads, seed=1)
    for _ in range(args.warmup):
        samp.step()
    t0 = time.perf_counter()
    done = 0.0
    for _ in range(args.steps):
        done += samp.step()
    dt = time.perf_counter() - t0
    v = done / dt
    sample = (f"1/64 of each matrix's output rows per step (2 of 128 rows of P^T G, m/64 rows of the weight delta "
              f"and NF4 weight apply) over the 7 matrices of the C2 block; params/s = 1/64 x 202.4M x steps / time")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * 202.4e6 / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD + " -- reference CPU algorithm (two-sided fp32 GaLore, per-tensor "
                                              "INT8, NF4 dequant + fp32 apply)", "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args):
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig, nf4_quantize
    from aethelstream_b200 import _lib
    from aethelstream_b200.sharding import allreduce_sqnorm_hook, setup_clip_group

    dev = torch.device("cuda", local)
    layer = rank  # weak scaling: one block per rank (round-robin layer ownership)
    specs = [(layer, name, m, n, RANK) for name, m, n in SHAPES]
    # C2 holds the projectors fixed (no gradient capture, no refresh inside the timed steps)
    cfg = GaLoreConfig(mode="b200", state_codec="dynamic", state_block=STATE_BLOCK,
                       layer_ranks=LayerRankConfig(), svd_refresh=False)
    opt = GaLoreOptimizer(cfg, specs, device=local)
    gen = torch.Generator(device=dev)
    weights = []
    for i, (name, m, n) in enumerate(SHAPES):
        gen.manual_seed(1000 * layer + i)
        w = torch.randn(m, n, generator=gen, device=dev) * 0.02
        weights.append(nf4_quantize(w))
        del w
    ring = []
    for parity in range(2):
        gs = []
        for i, (name, m, n) in enumerate(SHAPES):
            gen.manual_seed(7919 * (parity + 1) + 100 * layer + i)
            gs.append((torch.randn(m, n, generator=gen, device=dev) * 1e-3).to(torch.bfloat16))
        ring.append(gs)
    keys = [(layer, name) for name, _, _ in SHAPES]
    stream = torch.cuda.current_stream()
    # One GPU: the squared norms and the clip come from one launch.  Several
    # GPUs: that launch also exchanges the local sum with the peer GPUs over
    # NVLink (peer clip group); if the group cannot be set up, an NCCL
    # all-reduce hook between the norm and Adam phases does it instead.
    hook = None
    clip_exchange = "local (one GPU)"
    if world > 1:
        if setup_clip_group(opt, timeout_s=5.0):
            clip_exchange = "peer memory: NVLink stores and acquire loads inside the squared-norm launch"
        else:
            hook = allreduce_sqnorm_hook()
            clip_exchange = "NCCL all-reduce hook (peer clip group unavailable)"

    def step(s):
        return opt.step_layer(keys, ring[s % 2], weights, sq_hook=hook)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler start
    opt.set_phase_timing(True)  # CUDA events at the phase boundaries, on this stream
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    h0 = time.perf_counter()
    for s in range(args.steps):
        step(s)
    host_ms = (time.perf_counter() - h0) * 1000.0 / args.steps  # enqueue time only (the loop does not wait)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    opt.set_phase_timing(False)
    n_timed, phase_ms = opt.phase_times()
    assert n_timed == args.steps, (n_timed, args.steps)
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    t = torch.tensor([ms] + [phase_ms[k] for k in opt.PHASES], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t[0].item()
    phase_ms = dict(zip(opt.PHASES, t[1:].tolist()))
    params_per_step = sum(m * n for _, m, n in SHAPES)
    value = params_per_step * world * args.steps / (ms / 1000.0)

    # ---- the same steps replayed from CUDA graphs (one per gradient-ring parity; N = 1,
    # where the step has no host callback): one graph launch per step instead of four
    graph_ms = None
    if world == 1:
        graphs = []
        for parity in range(2):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                opt.step_layer(keys, ring[parity], weights)
            graphs.append(gr)
        for s in range(args.warmup):
            graphs[s % 2].replay()
        torch.cuda.synchronize()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for s in range(args.steps):
            graphs[s % 2].replay()
        g1.record(stream)
        torch.cuda.synchronize()
        graph_ms = g0.elapsed_time(g1) / args.steps
        del graphs

    # ---- end to end through the public API: pinned host grads -> device, step, clip -> host
    host_grads = [g.cpu().pin_memory() for g in ring[0]]
    dev_grads = [torch.empty_like(g) for g in ring[0]]
    clip_host = torch.empty(1, dtype=torch.float32).pin_memory()
    h2d = sum(g.numel() * g.element_size() for g in host_grads)
    k_e2e = max(3, min(args.steps, 20))

    def e2e_step():
        for hg, dg in zip(host_grads, dev_grads):
            dg.copy_(hg, non_blocking=True)
        clip = opt.step_layer(keys, dev_grads, weights, sq_hook=hook)
        clip_host.copy_(clip, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return float(clip_host[0])

    e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(k_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = params_per_step * world * k_e2e / (float(e2e_ms.item()) / 1000.0)
    dev_err = _lib.device_error_bits(local)
    if dev_err:
        raise RuntimeError(f"a bounded device wait gave up during the bench (error bits {dev_err:#x})")

    if rank == 0:
        hbm, tflops, tflops_sus, peak_kind = load_peaks()
        alg = algorithmic()
        kb = kernel_bytes()
        per_ms = {k: v / args.steps for k, v in phase_ms.items()}
        gbs = {k: kb[k] / (per_ms[k] / 1000.0) / 1e9 for k in opt.PHASES}
        traffic = load_traffic() if args.config == "c2" else {}  # the committed capture is of C2
        dom = max(opt.PHASES, key=lambda k: per_ms[k])
        achieved = gbs[dom]
        step_s = ms / args.steps / 1000.0
        total_bytes = alg["proj_bytes"] + alg["apply_bytes"]
        total_flops = alg["proj_flops"] + alg["apply_flops"]
        ideal_s = max(total_bytes / (hbm * 1e9), total_flops / (tflops_sus * 1e12))
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) NF4 weights, N(0,1e-3) bf16 grads)",
            "config": {"workload": WORKLOAD, "params_per_gpu_step": params_per_step, "rank": RANK,
                       "state": "int8 dynamic-map, 2048-element blocks", "parallelism": f"layer-sharded x{world}",
                       "clip_exchange": clip_exchange,
                       "l2": (f"inputs larger than L2 ({2 * params_per_step / 1e6:.0f} MB of bf16 gradients per "
                              "step, 2-deep ring)") if 2 * params_per_step > 126e6 else
                             f"inputs smaller than L2 ({2 * params_per_step / 1e6:.0f} MB of bf16 gradients)"},
            "roofline": {"bound": "hbm", "kernel": KERNEL_NAMES[dom], "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": traffic.get(f"{dom}_bytes_per_launch"),
                         "algorithmic_bytes_per_launch": kb[dom], "launch_ms": per_ms[dom],
                         "peak_kind": peak_kind},
            "roofline_step": {"algorithmic_bytes": total_bytes, "algorithmic_flops": total_flops,
                              "ideal_ms": ideal_s * 1000.0, "measured_ms": step_s * 1000.0,
                              "frac": ideal_s / step_s,
                              "phase_ms": per_ms, "phase_gbs": gbs, "phase_bytes": kb,
                              "host_enqueue_ms_per_step": host_ms, "graph_replay_ms_per_step": graph_ms},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                    "steps": k_e2e},
            # per step: grouped projection, sqnorm + clip (+ peer exchange), grouped Adam, grouped apply;
            # the NCCL hook adds the clip kernel
            "gpu_launches": (5 if hook is not None else 4) * args.steps,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            v, dt = cpu_baseline(1.0 / 128, 1)
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": 1, "kind": "port",
                                    "sample": "reference CPU algorithm (oracle port), 1/128 of each matrix's output "
                                              f"rows over the 7 C2 matrices, single thread, {dt:.1f} s"}
        print(json.dumps(line), flush=True)
    opt.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    global SHAPES, WORKLOAD
    SHAPES = CONFIGS[args.config]["shapes"]
    WORKLOAD = CONFIGS[args.config]["workload"]
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
