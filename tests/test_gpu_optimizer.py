"""The optimizer handle (OptimizerBackend mirror) on the GPU against the
oracle.

REF mode reproduces the reference's CPU loops: projections, Adam state,
weight delta and sqnorm are compared bit for bit.  B200 mode (tcgen05, bf16)
is compared within the stated tolerances, with the INT8 state codes and the
NF4 requantisation compared bit for bit on identical fp32 inputs.
"""
import numpy as np
import pytest
import torch

from tests._gpu import DEV, dev, host, rel_fro

pytestmark = pytest.mark.gpu


def _opt(mode, specs, **kw):
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig
    cfg = GaLoreConfig(mode=mode, layer_ranks=LayerRankConfig(**kw.pop("ranks", {})), **kw)
    return GaLoreOptimizer(cfg, specs, device=0)


# --------------------------------------------------------------------------- REF
def test_ref_mode_matches_cpu_reference_bitexact(oracle):
    specs = [(0, "d_wq", 64, 64), (0, "d_wg", 96, 64), (1, "d_wd", 64, 96)]
    opt = _opt("ref", specs)
    rng = np.random.default_rng(21)
    for li, name, m, n in specs:
        r = oracle.rank_for_param(name, m, n)
        P, Q = opt.get_projector(li, name)
        p_ref = oracle.init_random_projection(m, r, li * 17)
        q_ref = oracle.init_random_projection(n, r, li * 31)
        assert np.array_equal(host(P), p_ref) and np.array_equal(host(Q), q_ref)
        # two micro-batches (project_and_accumulate sums them, optimizer.rs:264-292)
        g1 = (rng.standard_normal((m, n)) * 1e-2).astype(np.float32)
        g2 = (rng.standard_normal((m, n)) * 1e-2).astype(np.float32)
        opt.project_and_accumulate(dev(g1), li, name)
        opt.project_and_accumulate(dev(g2), li, name)
        acc_ref = oracle.project_forward(g1, p_ref, q_ref, m, n, r).ravel()
        acc_ref = (acc_ref + oracle.project_forward(g2, p_ref, q_ref, m, n, r).ravel()).astype(np.float32)
        assert np.array_equal(host(opt.get_accum(li, name)), acc_ref)
        assert opt.lowrank_grad_sqnorm(li, name) == oracle.sqnorm_f64(acc_ref) or \
            abs(opt.lowrank_grad_sqnorm(li, name) - oracle.sqnorm_f64(acc_ref)) <= 1e-15 * oracle.sqnorm_f64(acc_ref)
        clip = 0.8
        opt.apply_update(li, name, clip)
        delta = opt.take_weight_delta(li, name)
        wd, nrm, m8, v8, sm, sv = oracle.galore_apply_update(acc_ref, p_ref, q_ref, np.zeros(r * r, np.int8),
                                                             np.zeros(r * r, np.int8), 1.0, 1.0, m, n, r, clip)
        gm8, gv8, gms, gvs = opt.get_state(li, name)
        assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8)
        assert host(gms)[0] == sm and host(gvs)[0] == sv
        assert np.array_equal(host(delta), wd)
        assert opt.take_weight_delta(li, name) is None
        opt.zero_accum(li, name)
        assert not host(opt.get_accum(li, name)).any()
    # unknown keys are ignored, as in the reference (optimizer.rs:270-291)
    opt.project_and_accumulate(torch.zeros(4, device=DEV), 9, "lm_head")
    assert opt.lowrank_grad_sqnorm(9, "lm_head") == 0.0
    opt.close()


def test_ref_mode_fp32_weight_inplace(oracle):
    m, n = 80, 48
    opt = _opt("ref", [(2, "d_wo", m, n)])
    r = oracle.rank_for_param("d_wo", m, n)
    rng = np.random.default_rng(22)
    g = (rng.standard_normal((m, n)) * 1e-2).astype(np.float32)
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    tw = dev(w)
    opt.project_and_accumulate(dev(g), 2, "d_wo")
    opt.apply_update(2, "d_wo", 1.0, weight=tw)
    p = oracle.init_random_projection(m, r, 34)
    q = oracle.init_random_projection(n, r, 62)
    acc = oracle.project_forward(g, p, q, m, n, r)
    wd, *_ = oracle.galore_apply_update(acc, p, q, np.zeros(r * r, np.int8), np.zeros(r * r, np.int8), 1.0, 1.0,
                                        m, n, r, 1.0)
    assert np.array_equal(host(tw), (w - wd).astype(np.float32))
    opt.close()


# --------------------------------------------------------------------------- B200
@pytest.mark.parametrize("m,n,r,codec", [(256, 128, 32, "linear"), (128, 384, 64, "linear"),
                                         (512, 512, 128, "dynamic"), (384, 256, 64, "dynamic"),
                                         (1024, 512, 512, "dynamic"), (512, 768, 384, "dynamic")])
def test_b200_step_matches_oracle(oracle, m, n, r, codec):
    from aethelstream_b200 import nf4_quantize
    rng = np.random.default_rng(m + n + r)
    name = "d_wq"
    opt = _opt("b200", [(3, name, m, n, r)], state_codec=codec)
    oc = oracle.CODEC_LINEAR if codec == "linear" else oracle.CODEC_DYNAMIC
    right = m >= n
    s = n if right else m
    l = m if right else n
    proj = oracle.init_random_projection(s, r, 3 * (31 if right else 17))
    proj_bf = oracle.bf16_round(proj)
    P, Q = opt.get_projector(3, name)
    assert np.array_equal(host(Q if right else P), proj_bf.reshape(s, r))
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    W = nf4_quantize(dev(w))
    wp, wa = host(W.packed), host(W.absmax)
    m8 = np.zeros(l * r, np.int8)
    v8 = np.zeros(l * r, np.int8)
    nb = (l * r + 2047) // 2048
    ms = np.full(nb, 1.0 if codec == "linear" else 0.0, np.float32)
    vs = ms.copy()
    for step in range(3):
        g = oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32))
        tg = dev(g).to(torch.bfloat16)
        opt.project_and_accumulate(tg, 3, name)
        acc = host(opt.get_accum(3, name))
        acc_ref = oracle.b2_project_accumulate(g, proj_bf, np.zeros(l * r, np.float32), m, n, r)
        assert rel_fro(acc, acc_ref) < 1e-5, step
        sq = opt.lowrank_grad_sqnorm(3, name)
        assert abs(sq - oracle.sqnorm_f64(acc)) <= 1e-12 * sq
        clip = float(oracle.clip_coeff(sq, 1.0))
        pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
        opt.apply_update(3, name, clip, weight=W, prequant_out=pre)
        opt.zero_accum(3, name)
        # state transition on the GPU's own accumulator: bit-exact
        n_ref, m8, v8, ms, vs = oracle.b2_adam_state(acc, m8, v8, ms, vs, 2048, oc, clip)
        gm8, gv8, gms, gvs = opt.get_state(3, name)
        assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8), step
        assert np.array_equal(host(gms), ms) and np.array_equal(host(gvs), vs), step
        # weight update: fp32 tolerance on the pre-quantisation values
        wp_ref, wa_ref, pre_ref, dw_ref = oracle.b2_apply_weight(n_ref, proj_bf, m, n, r, wp, wa, 1e-3)
        w_old = oracle.nf4_dequant_f32(wp, wa, m * n)
        upd_gpu = host(pre).ravel() - w_old
        upd_ref = pre_ref - w_old
        assert rel_fro(upd_gpu, upd_ref) < 1e-5, step
        # NF4 requantisation bit-exact on the GPU's own pre-quant values
        p_chk, a_chk = oracle.nf4_requant(host(pre).ravel())
        wp, wa = host(W.packed), host(W.absmax)
        assert np.array_equal(wp, p_chk) and np.array_equal(wa, a_chk), step
    opt.close()


@pytest.mark.parametrize("m,n", [(4096, 1024), (1024, 4096)])
def test_b200_projection_split_k_accumulates(oracle, m, n):
    """Shapes with few row tiles make the grouped projection split K across
    CTAs (partials added with TMA reduce-add); two calls accumulate."""
    r = 128
    opt = _opt("b200", [(0, "d_wq", m, n, r)])
    rng = np.random.default_rng(m)
    right = m >= n
    s, l = (n, m) if right else (m, n)
    P, Q = opt.get_projector(0, "d_wq")
    proj = host(Q if right else P)
    assert np.array_equal(proj, oracle.bf16_round(oracle.init_random_projection(s, r, 0)))  # layer 0: seed 0
    acc_ref = np.zeros(l * r, np.float32)
    for _ in range(2):
        g = oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32))
        opt.project_and_accumulate(dev(g).to(torch.bfloat16), 0, "d_wq")
        acc_ref = oracle.b2_project_accumulate(g, proj, acc_ref, m, n, r)
    assert rel_fro(host(opt.get_accum(0, "d_wq")), acc_ref) < 1e-5
    opt.close()


def test_b200_fused_layer_step_equals_sequential(oracle):
    from aethelstream_b200 import nf4_quantize
    specs = [(0, "d_wq", 256, 256, 64), (0, "d_wg", 512, 256, 64), (0, "d_wd", 256, 512, 64)]
    rng = np.random.default_rng(31)
    grads = [oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)) for _, _, m, n, _ in specs]
    ws = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for _, _, m, n, _ in specs]
    results = []
    for fused in (False, True):
        opt = _opt("b200", specs, max_grad_norm=0.01)
        W = [nf4_quantize(dev(w)) for w in ws]
        G = [dev(g).to(torch.bfloat16) for g in grads]
        if fused:
            clip = opt.step_layer([(li, nm) for li, nm, *_ in specs], G, W)
            clip = float(host(clip)[0])
        else:
            for (li, nm, *_), g in zip(specs, G):
                opt.project_and_accumulate(g, li, nm)
            sq = sum(opt.lowrank_grad_sqnorm(li, nm) for li, nm, *_ in specs)
            clip = float(oracle.clip_coeff(sq, 0.01))
            for (li, nm, *_), w in zip(specs, W):
                opt.apply_update(li, nm, clip, weight=w)
                opt.zero_accum(li, nm)
        assert clip < 1.0
        results.append((clip, [host(w.packed) for w in W], [host(w.absmax) for w in W],
                        [host(x) for li, nm, *_ in specs for x in opt.get_state(li, nm)]))
        opt.close()
    (c0, p0, a0, s0), (c1, p1, a1, s1) = results
    assert c0 == c1
    for x, y in zip(p0 + a0 + s0, p1 + a1 + s1):
        assert np.array_equal(x, y)


def test_b200_step_with_hook_equals_fused_clip(oracle):
    """With a squared-norm hook the step runs norms, hook and clip as separate
    launches; without one the norm kernel also writes the clip.  Same results,
    and the per-phase timing records every step."""
    from aethelstream_b200 import nf4_quantize
    specs = [(0, "d_wq", 256, 512, 64), (0, "d_wk", 512, 256, 64)]
    rng = np.random.default_rng(47)
    grads = [oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)) for _, _, m, n, _ in specs]
    ws = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for _, _, m, n, _ in specs]
    results = []
    for use_hook in (False, True):
        opt = _opt("b200", specs, max_grad_norm=0.01)
        opt.set_phase_timing(True)
        W = [nf4_quantize(dev(w)) for w in ws]
        G = [dev(g).to(torch.bfloat16) for g in grads]
        seen = []
        hook = (lambda sq: seen.append(float(sq.sum()))) if use_hook else None
        clips = [float(host(opt.step_layer([(li, nm) for li, nm, *_ in specs], G, W, sq_hook=hook))[0])
                 for _ in range(3)]
        steps, ms = opt.phase_times()
        assert steps == 3
        assert all(v > 0.0 for v in ms.values()), ms
        assert opt.phase_times()[0] == 0
        if use_hook:
            assert len(seen) == 3
        results.append((clips, [host(w.packed) for w in W], [host(w.absmax) for w in W],
                        [host(x) for li, nm, *_ in specs for x in opt.get_state(li, nm)]))
        opt.close()
    (c0, p0, a0, s0), (c1, p1, a1, s1) = results
    assert c0 == c1 and c0[0] < 1.0
    for x, y in zip(p0 + a0 + s0, p1 + a1 + s1):
        assert np.array_equal(x, y)


def test_b200_apply_nonfinite_blocks(oracle):
    """NF4 blocks whose weights turn NaN or infinite are requantised as the
    reference's quantiser does (absmax NaN or inf, codes from the exact
    argmin), without the fast classifier's table lookup; the other blocks of
    the same tiles are unaffected."""
    from aethelstream_b200 import nf4_quantize
    m, n, r = 256, 512, 64
    rng = np.random.default_rng(61)
    opt = _opt("b200", [(0, "d_wq", m, n, r)])
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    W = nf4_quantize(dev(w))
    W.absmax[5] = float("nan")         # every weight NaN
    W.absmax[9] = float("inf")         # +-inf, and NaN where the code is 0.0
    W.packed[13 * 32:14 * 32] = 0xFF   # code 1.0 throughout ...
    W.absmax[13] = float("inf")        # ... so every weight is +inf
    W.packed[17 * 32:18 * 32] = 0xFF
    W.absmax[17] = 1e38                # large but finite
    g = oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32))
    opt.project_and_accumulate(dev(g).to(torch.bfloat16), 0, "d_wq")
    pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
    opt.apply_update(0, "d_wq", 1.0, weight=W, prequant_out=pre)
    pre_h = host(pre).ravel()
    assert np.isnan(pre_h[5 * 64:6 * 64]).all()
    assert np.isposinf(pre_h[13 * 64:14 * 64]).all()
    p_chk, a_chk = oracle.nf4_requant(pre_h)
    a_gpu = host(W.absmax)
    assert np.isnan(a_gpu[5]) and np.isnan(a_gpu[9]) and np.isposinf(a_gpu[13]) and np.isfinite(a_gpu[17])
    assert np.array_equal(host(W.packed), p_chk)
    assert np.array_equal(a_gpu.view(np.uint32), a_chk.view(np.uint32))
    assert (host(W.packed)[5 * 32:6 * 32] == 0).all() and (host(W.packed)[13 * 32:14 * 32] == 0).all()
    opt.close()


def test_b200_apply_requant_bitexact_large(oracle):
    """The fused requantisation at a size where hundreds of updated weights land
    next to a decision midpoint (the exact repair path), bit-exact against the
    reference quantiser on the kernel's own pre-quantisation values."""
    from aethelstream_b200 import nf4_quantize
    m, n, r = 2048, 4096, 128
    rng = np.random.default_rng(62)
    opt = _opt("b200", [(0, "d_wq", m, n, r)])
    W = nf4_quantize(dev((rng.standard_normal((m, n)) * 0.02).astype(np.float32)))
    pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
    for step in range(2):
        g = (torch.randn(m, n, device=DEV) * 1e-3).to(torch.bfloat16)
        opt.project_and_accumulate(g, 0, "d_wq")
        opt.apply_update(0, "d_wq", 1.0, weight=W, prequant_out=pre)
        opt.zero_accum(0, "d_wq")
        pre_h = host(pre).ravel()
        p_chk, a_chk = oracle.nf4_requant(pre_h)
        assert np.array_equal(host(W.packed), p_chk), step
        assert np.array_equal(host(W.absmax).view(np.uint32), a_chk.view(np.uint32)), step
    # the repair path ran: weights within the near window of a midpoint
    codes = oracle.NF4_CODES
    mids = ((codes[:-1] + codes[1:]) * np.float32(0.5)).astype(np.float32)
    xn = (pre_h.reshape(-1, 64) / np.maximum(a_chk, 1e-8)[:, None]).ravel()
    near = np.abs(xn[:, None] - mids[None, :]).min(axis=1) < 1.5e-6
    assert near.sum() > 20, near.sum()
    opt.close()


def test_b200_step_cuda_graph_replay_equals_eager(oracle):
    """The fused step records into a CUDA graph (no host synchronisation, no
    allocation, device-side counters); replaying it equals running it eagerly,
    bit for bit.  Phase timing is skipped while capturing, and a capture with
    the gradient-driven subspace refresh on is refused."""
    from aethelstream_b200 import _lib, nf4_quantize
    specs = [(0, "d_wq", 256, 512, 64), (0, "d_wg", 512, 256, 64)]
    keys = [(li, nm) for li, nm, *_ in specs]
    rng = np.random.default_rng(71)
    ring = [[dev((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)).to(torch.bfloat16)
             for _, _, m, n, _ in specs] for _ in range(2)]
    w0 = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for _, _, m, n, _ in specs]
    results = []
    for use_graph in (False, True):
        opt = _opt("b200", specs, max_grad_norm=0.01, svd_refresh=False)
        W = [nf4_quantize(dev(w)) for w in w0]
        clips = []
        if use_graph:
            static = [torch.empty_like(g) for g in ring[0]]
            for sg, g in zip(static, ring[0]):
                sg.copy_(g)
            graph = torch.cuda.CUDAGraph()
            opt.set_phase_timing(True)
            with torch.cuda.graph(graph):
                clip = opt.step_layer(keys, static, W)
            opt.set_phase_timing(False)
            assert opt.phase_times()[0] == 0  # nothing recorded during capture
            for s in range(4):
                for sg, g in zip(static, ring[s % 2]):
                    sg.copy_(g)
                graph.replay()
                clips.append(float(host(clip)[0]))
            del graph
        else:
            for s in range(4):
                clips.append(float(host(opt.step_layer(keys, ring[s % 2], W))[0]))
        results.append((clips, [host(w.packed) for w in W], [host(w.absmax) for w in W],
                        [host(x) for li, nm, *_ in specs for x in opt.get_state(li, nm)]))
        opt.close()
    (c0, p0, a0, s0), (c1, p1, a1, s1) = results
    assert c0 == c1 and c0[0] < 1.0
    for x, y in zip(p0 + a0 + s0, p1 + a1 + s1):
        assert np.array_equal(x, y)
    # the refresh schedule cannot be replayed: capture is refused with it on
    opt = _opt("b200", specs, svd_refresh=True)
    W = [nf4_quantize(dev(w)) for w in w0]
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(_lib.AethError):
        with torch.cuda.graph(graph):
            opt.step_layer(keys, ring[0], W)
    opt.close()
