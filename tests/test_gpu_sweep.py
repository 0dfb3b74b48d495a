"""The streamed whole-model step on the GPU: per-layer grouped projections
(aeth_galore_project_layer, as doublepass's backward hands each layer's
gradients to the optimizer, backward.rs:509-521) followed by one finishing
call (aeth_galore_finish_step: the exact global clip over every parameter,
then Adam and the weight write, hook.rs:115-203), and the exact bf16-term
path for fp32 / f16 gradients."""
import numpy as np
import pytest
import torch

from tests._gpu import DEV, dev, host, rel_fro

pytestmark = pytest.mark.gpu


def _opt(specs, **kw):
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer
    cfg = GaLoreConfig(mode="b200", state_codec=kw.pop("state_codec", "dynamic"), svd_refresh=False, **kw)
    return GaLoreOptimizer(cfg, specs, device=0)


def _model(layers, shapes, r):
    return [(li, nm, m, n, r) for li in range(layers) for nm, m, n in shapes]


def _snapshot(opt, specs, W):
    return ([host(w.packed) for w in W] + [host(w.absmax) for w in W] +
            [host(x) for li, nm, *_ in specs for x in opt.get_state(li, nm)])


def test_streamed_layers_equal_one_step(oracle):
    """project_layer for each of three layers, then finish_step over all nine
    parameters, gives the bits of one aeth_galore_step over the same nine."""
    from aethelstream_b200 import nf4_quantize
    shapes = [("d_wq", 256, 256), ("d_wg", 512, 256), ("d_wd", 256, 512)]
    specs = _model(3, shapes, 64)
    keys = [(li, nm) for li, nm, *_ in specs]
    rng = np.random.default_rng(5)
    grads = [oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)) for *_, m, n, _ in specs]
    ws = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for *_, m, n, _ in specs]
    out = []
    for streamed in (False, True):
        opt = _opt(specs, max_grad_norm=0.02)
        W = [nf4_quantize(dev(w)) for w in ws]
        G = [dev(g).to(torch.bfloat16) for g in grads]
        clips = []
        for _ in range(2):
            if streamed:
                for li in range(3):
                    sel = [i for i, k in enumerate(keys) if k[0] == li]
                    opt.project_layer([keys[i] for i in sel], [G[i] for i in sel])
                clip = opt.finish_step(keys, W)
            else:
                clip = opt.step_layer(keys, G, W)
            clips.append(float(host(clip)[0]))
        out.append((clips, _snapshot(opt, specs, W)))
        opt.close()
    (c0, s0), (c1, s1) = out
    assert c0 == c1 and c0[0] < 1.0
    for x, y in zip(s0, s1):
        assert np.array_equal(x, y)


def test_finish_step_clip_over_many_parameters(oracle):
    """A whole model's clip in one squared-norm launch: 40 parameters (above the
    single-layer launch's capacity of 16), the global clip equal to the
    reference's formula over the accumulators, the INT8 state bit-exact."""
    from aethelstream_b200 import nf4_quantize
    shapes = [("d_wq", 256, 256), ("d_wk", 128, 256), ("d_wv", 128, 256), ("d_wo", 256, 256),
              ("d_wg", 512, 256), ("d_wu", 512, 256), ("d_wd", 256, 512), ("d_wx", 256, 256)]
    r = 64
    specs = _model(5, shapes, r)
    assert len(specs) == 40
    keys = [(li, nm) for li, nm, *_ in specs]
    rng = np.random.default_rng(6)
    opt = _opt(specs, max_grad_norm=0.05)
    W = [nf4_quantize(dev((rng.standard_normal((m, n)) * 0.02).astype(np.float32))) for *_, m, n, _ in specs]
    for li in range(5):
        sel = [i for i, k in enumerate(keys) if k[0] == li]
        G = [dev(oracle.bf16_round((rng.standard_normal((specs[i][2], specs[i][3])) * 1e-3).astype(np.float32)))
             .to(torch.bfloat16) for i in sel]
        opt.project_layer([keys[i] for i in sel], G)
    accs = [host(opt.get_accum(li, nm)) for li, nm in keys]
    sq = sum(oracle.sqnorm_f64(a) for a in accs)
    clip_ref = float(oracle.clip_coeff(sq, 0.05))
    clip = float(host(opt.finish_step(keys, W))[0])
    assert clip < 1.0
    assert abs(clip - clip_ref) <= 2e-7 * clip_ref, (clip, clip_ref)
    for (li, nm), a, (*_, m, n, _) in zip(keys, accs, specs):
        l = max(m, n)
        nb = (l * r) // 2048
        z8 = np.zeros(l * r, np.int8)
        zs = np.zeros(nb, np.float32)
        _, m8, v8, ms, vs = oracle.b2_adam_state(a, z8, z8, zs, zs, 2048, oracle.CODEC_DYNAMIC, clip)
        gm8, gv8, gms, gvs = opt.get_state(li, nm)
        assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8)
        assert np.array_equal(host(gms), ms) and np.array_equal(host(gvs), vs)
        assert not host(opt.get_accum(li, nm)).any()
    opt.close()


def test_streamed_step_graph_replay_equals_eager(oracle):
    """The whole streamed step (three project_layer calls and finish_step)
    records into one CUDA graph; replays equal eager calls bit for bit."""
    from aethelstream_b200 import nf4_quantize
    shapes = [("d_wq", 256, 512), ("d_wg", 512, 256)]
    specs = _model(3, shapes, 64)
    keys = [(li, nm) for li, nm, *_ in specs]
    rng = np.random.default_rng(7)
    ring = [[dev((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)).to(torch.bfloat16)
             for _, m, n in shapes] for _ in range(2)]
    w0 = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for *_, m, n, _ in specs]

    def step(opt, W, s):
        for li in range(3):
            opt.project_layer([k for k in keys if k[0] == li], ring[(s + li) % 2])
        return opt.finish_step(keys, W)

    out = []
    for use_graph in (False, True):
        opt = _opt(specs, max_grad_norm=0.02)
        W = [nf4_quantize(dev(w)) for w in w0]
        clips = []
        if use_graph:
            graphs = []
            for parity in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    clip = step(opt, W, parity)
                graphs.append((g, clip))
            for s in range(4):
                graphs[s % 2][0].replay()
                clips.append(float(host(graphs[s % 2][1])[0]))
            del graphs
        else:
            for s in range(4):
                clips.append(float(host(step(opt, W, s % 2))[0]))
        out.append((clips, _snapshot(opt, specs, W)))
        opt.close()
    (c0, s0), (c1, s1) = out
    assert c0 == c1
    for x, y in zip(s0, s1):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("dtype", ["f32", "f16"])
@pytest.mark.parametrize("m,n", [(512, 256), (256, 768)])
@pytest.mark.parametrize("declared", [True, False])
def test_split_gradient_projection(oracle, dtype, m, n, declared):
    """fp32 / f16 gradients are not narrowed to bf16: their exact bf16 terms are
    projected together, so the accumulator matches the oracle's f64 product of
    the unrounded gradient with the bf16 projector to fp32 accuracy, and the
    bf16-narrowed result is measurably worse."""
    r = 64
    tdt = torch.float32 if dtype == "f32" else torch.float16
    opt = _opt([(0, "d_wq", m, n, r)], grad_dtype=dtype if declared else "bf16")
    right = m >= n
    s, l = (n, m) if right else (m, n)
    P, Q = opt.get_projector(0, "d_wq")
    proj = host(Q if right else P)
    rng = np.random.default_rng(m + n)
    acc_ref = np.zeros(l * r, np.float32)
    for _ in range(2):
        g = (rng.standard_normal((m, n)) * 1e-3).astype(np.float32)
        tg = dev(g).to(tdt)
        g_exact = host(tg.float())
        opt.project_and_accumulate(tg, 0, "d_wq")
        acc_ref = oracle.b2_project_accumulate(g_exact, proj, acc_ref, m, n, r)
    acc = host(opt.get_accum(0, "d_wq"))
    err = rel_fro(acc, acc_ref)
    assert err < 1e-6, err
    narrowed = oracle.b2_project_accumulate(oracle.bf16_round(g_exact), proj, np.zeros(l * r, np.float32), m, n, r)
    single = oracle.b2_project_accumulate(g_exact, proj, np.zeros(l * r, np.float32), m, n, r)
    assert rel_fro(narrowed, single) > 10 * err
    opt.close()


def test_split_gradient_capture(oracle):
    """A declared fp32 gradient dtype sets the split buffers up at construction,
    so the step records into a CUDA graph and replays equal eager steps; an
    undeclared fp32 gradient is refused while capturing (the buffers would
    need an allocation)."""
    from aethelstream_b200 import _lib, nf4_quantize
    m, n, r = 512, 256, 64
    keys = [(0, "d_wq")]
    rng = np.random.default_rng(8)
    g = dev((rng.standard_normal((m, n)) * 1e-3).astype(np.float32))
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    out = []
    for use_graph in (False, True):
        opt = _opt([(0, "d_wq", m, n, r)], grad_dtype="f32")
        W = [nf4_quantize(dev(w))]
        if use_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                opt.step_layer(keys, [g], W)
            for _ in range(3):
                graph.replay()
            del graph
        else:
            for _ in range(3):
                opt.step_layer(keys, [g], W)
        out.append([host(W[0].packed), host(W[0].absmax)] + [host(x) for x in opt.get_state(0, "d_wq")])
        opt.close()
    for x, y in zip(*out):
        assert np.array_equal(x, y)
    opt = _opt([(0, "d_wq", m, n, r)])
    W = [nf4_quantize(dev(w))]
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(_lib.AethError):
        with torch.cuda.graph(graph):
            opt.step_layer(keys, [g], W)
    opt.close()
