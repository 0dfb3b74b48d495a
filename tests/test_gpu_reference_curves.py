"""The product's REF mode driven through the reference's own GaLore training
run, against the losses the reference recorded.

The run is the one galore/tests/test_galore_theorem_38.rs and
test_galore_scale_independence.rs make: a 2-layer toy transformer whose
gradients come, step by step, from the CPU restatement of its model
(oracle.ToyModel, test infrastructure; it only supplies the gradients and
applies the weight deltas), while every optimizer operation -- projection and
accumulation, squared norms, Adam with the per-tensor INT8 state, the
back-projection and the learning-rate rule -- runs on the GPU through the
library (GaLoreOptimizer in REF mode with the exact-order products).

The runs here are the three recorded runs whose subspace refresh reached no
matrix (their first refresh job failed; tests/test_oracle_reference_curves.py),
so the library's refresh is off.  The losses equal the oracle's restatement of
the same run bit for bit over all 32 recorded steps, and the recorded losses
bit for bit over the steps where the oracle does.  The run's full-rank AdamW
baseline goes through doublepass_galore_apply the same way.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from oracle.galore_optimizer import RECORDED_RUNS, global_clip, run_recorded
from tests._gpu import dev, host, ptr
from tests.test_oracle_reference_curves import AGREEMENT

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
STEPS = 32


@pytest.fixture(scope="module")
def lib():
    from aethelstream_b200 import _lib
    return _lib.load()


@pytest.fixture(scope="module")
def curves():
    with open(os.path.join(HERE, "golden", "galore_curves.json")) as f:
        return {k: np.array(v, np.float32) for k, v in json.load(f).items() if not k.startswith("_")}


@pytest.mark.parametrize("run", ["theorem_38/galore_periodic_200", "scale_independence/no_rank_division",
                                 "scale_independence/with_rank_division"])
def test_ref_mode_reproduces_the_recorded_run(curves, run):
    from aethelstream_b200 import AdamWConfig, GaLoreConfig, GaLoreOptimizer, LayerRankConfig
    cfg = RECORDED_RUNS[run]
    model = O.ToyModel(*cfg["model"])
    specs = model.param_specs()
    gcfg = GaLoreConfig(mode="ref", layer_ranks=LayerRankConfig(*cfg["layer_ranks"]),
                        switch_interval=cfg["switch_interval"], svd_refresh=False, max_grad_norm=1.0,
                        adam=AdamWConfig(lr=cfg["lr"], scale_lr_by_rank=cfg["scale_lr_by_rank"]))
    opt = GaLoreOptimizer(gcfg, specs, device=0)
    losses = []
    try:
        for s in range(STEPS):
            loss, grads = model.step()
            for li in reversed(range(model.nl)):  # the backward's hook order, last layer first
                for name in model.NAMES:
                    opt.project_and_accumulate(dev(grads[(li, name)]), li, name)
            clip = global_clip([opt.lowrank_grad_sqnorm(li, nm) for (li, nm, _, _) in specs])
            for (li, nm, _, _) in specs:
                opt.apply_update(li, nm, float(clip))
                opt.zero_accum(li, nm)
            for (li, nm, m, n) in specs:
                model.apply_delta(li, nm, host(opt.take_weight_delta(li, nm)))
            opt.notify_step(s + 1)
            losses.append(np.float32(loss))
    finally:
        opt.close()
    losses = np.array(losses, np.float32)
    oracle_losses, _ = run_recorded(run, STEPS)
    assert np.array_equal(losses, oracle_losses), np.flatnonzero(losses != oracle_losses)
    exact = AGREEMENT[run][0]
    assert np.array_equal(losses[:exact], curves[run][:exact])


def test_full_rank_adam_reproduces_the_recorded_baseline(curves, lib):
    """The theorem-3.8 run's AdamW baseline with every update by the library's
    doublepass_galore_apply (step 0: StandardAdamW's update without bias
    correction) on device-resident weights and moments."""
    import torch
    cfg = RECORDED_RUNS["theorem_38/adamw"]
    model = O.ToyModel(*cfg["model"])
    specs = model.param_specs()
    state = {(li, nm): [torch.zeros(m * n, dtype=torch.float32, device="cuda:0") for _ in range(3)]
             for (li, nm, m, n) in specs}  # m, v, full-gradient accumulator
    losses = []
    for s in range(STEPS):
        loss, grads = model.step()
        for li in reversed(range(model.nl)):
            for name in model.NAMES:
                state[(li, name)][2] += dev(grads[(li, name)].ravel())
        clip = global_clip([O.sqnorm_f64(host(state[(li, nm)][2])) for (li, nm, _, _) in specs])
        for (li, nm, m, n) in specs:
            mm, vv, acc = state[(li, nm)]
            w = torch.zeros(m * n, dtype=torch.float32, device="cuda:0")  # 0 - delta = -delta exactly
            lib.doublepass_galore_apply(ptr(w), ptr(acc), ptr(mm), ptr(vv), float(clip), 0.9, 0.999, 1e-8, cfg["lr"],
                                        m * n, 0)
            assert lib.aeth_last_error() == 0
            model.apply_delta(li, nm, -host(w))
            acc.zero_()
        losses.append(np.float32(loss))
    losses = np.array(losses, np.float32)
    oracle_losses, _ = run_recorded("theorem_38/adamw", STEPS)
    assert np.array_equal(losses, oracle_losses), np.flatnonzero(losses != oracle_losses)
    exact = AGREEMENT["theorem_38/adamw"][0]
    assert np.array_equal(losses[:exact], curves["theorem_38/adamw"][:exact])
