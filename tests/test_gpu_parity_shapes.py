"""Parity of the whole step at the shapes BASELINE names, against the oracle.

* C1 exactly as stated: one 4096 x 4096 weight, W ~ N(0, 0.02) from seed 0
  stored NF4, an fp32 gradient N(0, 1e-3) from seed 1, the projector the Q
  factor of a Gaussian 4096 x 128 (seed 2), Adam 0.9 / 0.999 / 1e-3 / 1e-8,
  INT8 dynamic-map state in 2048-element blocks from zero;
* one 11008 x 4096 and one 4096 x 11008 matrix of C2 (bf16 gradients, r 128);
* rank 512 (C4), whose projection runs as two 256-column slices of R;
* a full layer of nine parameters -- the seven matrices plus the 1 x d
  RMS-norm vectors d_rms1_w / d_rms2_w whose rank clamps to 1
  (galore/tests/common/mod.rs:73-89, doublepass/src/backward.rs:512-520) --
  in B200 mode and in REF mode.

Tolerances (BASELINE): updated weights within 1e-5 relative (fp32) before
requantisation; INT8 codes and scales bit-exact on the GPU's own accumulator
and clip; NF4 requantisation bit-exact on the GPU's own pre-quantisation
values.  The projection of an fp32 gradient (its exact bf16 terms) within
1e-5 of the oracle's f64 product."""
import numpy as np
import pytest
import torch

from tests._gpu import DEV, dev, host, rel_fro

pytestmark = pytest.mark.gpu


def _opt(mode, specs, **kw):
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig
    cfg = GaLoreConfig(mode=mode, layer_ranks=LayerRankConfig(**kw.pop("ranks", {})), svd_refresh=False, **kw)
    return GaLoreOptimizer(cfg, specs, device=0)


def _check_b200_param(oracle, opt, li, name, m, n, r, g_exact, acc_gpu, clip, wp0, wa0, pre, W, lr=1e-3,
                      codec="dynamic", wd=0.0):
    """One parameter after one step from zero state: projection, INT8 state,
    weight update and requantisation against the oracle."""
    right = m >= n
    s, l = (n, m) if right else (m, n)
    P, Q = opt.get_projector(li, name)
    proj = host(Q if right else P)
    acc_ref = oracle.b2_project_accumulate(g_exact, proj, np.zeros(l * r, np.float32), m, n, r)
    assert rel_fro(acc_gpu, acc_ref) < 1e-5, (name, rel_fro(acc_gpu, acc_ref))
    nb = (l * r + 2047) // 2048
    oc = oracle.CODEC_DYNAMIC if codec == "dynamic" else oracle.CODEC_LINEAR
    z = np.zeros(nb, np.float32) if codec == "dynamic" else np.ones(nb, np.float32)
    n_ref, m8, v8, ms, vs = oracle.b2_adam_state(acc_gpu, np.zeros(l * r, np.int8), np.zeros(l * r, np.int8), z, z,
                                                 2048, oc, clip)
    gm8, gv8, gms, gvs = opt.get_state(li, name)
    assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8), name
    assert np.array_equal(host(gms), ms) and np.array_equal(host(gvs), vs), name
    _, _, pre_ref, _ = oracle.b2_apply_weight(n_ref, proj, m, n, r, wp0, wa0, lr, wd)
    w_old = oracle.nf4_dequant_f32(wp0, wa0, m * n)
    pre_h = host(pre).ravel()
    assert rel_fro(pre_h - w_old, pre_ref - w_old) < 1e-5, (name, rel_fro(pre_h - w_old, pre_ref - w_old))
    p_chk, a_chk = oracle.nf4_requant(pre_h)
    assert np.array_equal(host(W.packed), p_chk), name
    assert np.array_equal(host(W.absmax).view(np.uint32), a_chk.view(np.uint32)), name
    return pre_ref


def test_c1_baseline_config(oracle):
    from aethelstream_b200 import nf4_quantize
    m = n = 4096
    r = 128
    w = (torch.randn(m, n, generator=torch.Generator().manual_seed(0)) * 0.02).numpy()
    g = (torch.randn(m, n, generator=torch.Generator().manual_seed(1)) * 1e-3).numpy()
    basis = torch.linalg.qr(torch.randn(n, r, generator=torch.Generator().manual_seed(2), dtype=torch.float64))[0]
    opt = _opt("b200", [(0, "d_wq", m, n, r)], state_codec="dynamic", grad_dtype="f32", init_projectors=False)
    opt.set_projector(0, "d_wq", Q=dev(basis.float().numpy()))
    W = nf4_quantize(dev(w))
    wp0, wa0 = host(W.packed), host(W.absmax)
    p_ref, a_ref = oracle.nf4_quantize(w)
    assert np.array_equal(wp0, p_ref) and np.array_equal(wa0, a_ref)
    opt.project_and_accumulate(dev(g), 0, "d_wq")
    acc = host(opt.get_accum(0, "d_wq"))
    sq = opt.lowrank_grad_sqnorm(0, "d_wq")
    clip = float(oracle.clip_coeff(sq, 1.0))
    pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
    opt.apply_update(0, "d_wq", clip, weight=W, prequant_out=pre)
    pre_ref = _check_b200_param(oracle, opt, 0, "d_wq", m, n, r, g, acc, clip, wp0, wa0, pre, W)
    # the output C1 names: the dequantised weight after the update, against the
    # oracle's own requantisation of its own pre-quantisation values.  The two
    # pre-quantisation values agree to ~1e-7 of the update, so a block's
    # absmax (its largest |w|) agrees to within an ulp or two, and a code
    # differs only where a weight sits that close to a decision midpoint.
    wq_ref, aq_ref = oracle.nf4_requant(pre_ref)
    a_gpu = host(W.absmax)
    assert np.abs(a_gpu - aq_ref).max() <= 1e-6 * np.abs(aq_ref).max()
    codes_gpu = np.stack([host(W.packed) >> 4, host(W.packed) & 15])
    codes_ref = np.stack([wq_ref >> 4, wq_ref & 15])
    flips = np.count_nonzero(codes_gpu != codes_ref)
    assert flips <= 1e-4 * m * n, flips
    w_gpu = oracle.nf4_dequant_f32(host(W.packed), a_gpu, m * n)
    w_ref = oracle.nf4_dequant_f32(wq_ref, aq_ref, m * n)
    assert rel_fro(w_gpu, w_ref) < 1e-3
    opt.close()


@pytest.mark.parametrize("m,n,r", [(11008, 4096, 128), (4096, 11008, 128), (1024, 8192, 512), (4096, 1024, 512)])
def test_large_shapes_against_oracle(oracle, m, n, r):
    """C2's rectangular matrices and C4's rank 512 (two 256-column slices of R
    in the projection, eight k-blocks per unit in the back-projection)."""
    from aethelstream_b200 import nf4_quantize
    rng = np.random.default_rng(m * 7 + n + r)
    opt = _opt("b200", [(1, "d_wg", m, n, r)], state_codec="dynamic")
    W = nf4_quantize(dev((rng.standard_normal((m, n), dtype=np.float32) * np.float32(0.02))))
    wp0, wa0 = host(W.packed), host(W.absmax)
    g = oracle.bf16_round(rng.standard_normal((m, n), dtype=np.float32) * np.float32(1e-3))
    opt.project_and_accumulate(dev(g).to(torch.bfloat16), 1, "d_wg")
    acc = host(opt.get_accum(1, "d_wg"))
    sq = opt.lowrank_grad_sqnorm(1, "d_wg")
    clip = float(oracle.clip_coeff(sq, 1.0))
    pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
    opt.apply_update(1, "d_wg", clip, weight=W, prequant_out=pre)
    _check_b200_param(oracle, opt, 1, "d_wg", m, n, r, g, acc, clip, wp0, wa0, pre, W)
    opt.close()


@pytest.mark.parametrize("wd", [0.0, 0.1])
def test_apply_specialisations_and_decay(oracle, wd):
    """The back-projection kernel is compiled per launch for the decoupled
    decay (adamw.rs:194-202) and for the optional fp32 outputs.  With
    prequant_out the update is checked against the oracle (decay included);
    the launch without it -- the one the streamed step runs -- must write the
    same NF4 codes and scales from the same state."""
    from aethelstream_b200 import AdamWConfig, nf4_quantize
    m, n, r = 1024, 8192, 512
    rng = np.random.default_rng(int(wd * 10) + 77)
    w0 = rng.standard_normal((m, n), dtype=np.float32) * np.float32(0.02)
    g = oracle.bf16_round(rng.standard_normal((m, n), dtype=np.float32) * np.float32(1e-3))
    out = []
    for with_pre in (True, False):
        opt = _opt("b200", [(1, "d_wq", m, n, r)], state_codec="dynamic", adam=AdamWConfig(weight_decay=wd))
        W = nf4_quantize(dev(w0))
        wp0, wa0 = host(W.packed), host(W.absmax)
        opt.project_and_accumulate(dev(g).to(torch.bfloat16), 1, "d_wq")
        acc = host(opt.get_accum(1, "d_wq"))
        clip = float(oracle.clip_coeff(opt.lowrank_grad_sqnorm(1, "d_wq"), 1.0))
        if with_pre:
            pre = torch.empty(m, n, dtype=torch.float32, device=DEV)
            opt.apply_update(1, "d_wq", clip, weight=W, prequant_out=pre)
            _check_b200_param(oracle, opt, 1, "d_wq", m, n, r, g, acc, clip, wp0, wa0, pre, W, wd=wd)
        else:
            opt.apply_update(1, "d_wq", clip, weight=W)
        out.append((host(W.packed), host(W.absmax).view(np.uint32)))
        opt.close()
    assert np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1])


LAYER = [("d_rms1_w", 1, 256), ("d_wq", 256, 256), ("d_wk", 128, 256), ("d_wv", 128, 256), ("d_wo", 256, 256),
         ("d_rms2_w", 1, 256), ("d_wg", 512, 256), ("d_wu", 512, 256), ("d_wd", 256, 512)]


def test_b200_full_layer_nine_parameters(oracle):
    """The nine parameters of a layer through the fused step, with the default
    LayerRankConfig ranks (attention 32, MLP 16, vectors 8 clamped to 1)."""
    from aethelstream_b200 import nf4_quantize
    specs = [(2, nm, m, n) for nm, m, n in LAYER]
    opt = _opt("b200", specs, state_codec="dynamic", max_grad_norm=0.05)
    ranks = [oracle.rank_for_param(nm, m, n) for nm, m, n in LAYER]
    assert ranks[0] == 1 and ranks[5] == 1 and ranks[1] == 32 and ranks[6] == 16
    for (li, nm, m, n), r in zip(specs, ranks):
        assert opt.param_info(li, nm).rank == r
    rng = np.random.default_rng(90)
    W = [nf4_quantize(dev((rng.standard_normal((m, n)) * 0.02).astype(np.float32))) for _, m, n in LAYER]
    w0 = [(host(x.packed), host(x.absmax)) for x in W]
    gs = [oracle.bf16_round((rng.standard_normal((m, n)) * 1e-3).astype(np.float32)) for _, m, n in LAYER]
    keys = [(li, nm) for li, nm, *_ in specs]
    opt.project_layer(keys, [dev(g).to(torch.bfloat16) for g in gs])
    accs = [host(opt.get_accum(li, nm)) for li, nm in keys]
    sq = sum(oracle.sqnorm_f64(a) for a in accs)
    pres = [torch.empty(m, n, dtype=torch.float32, device=DEV) for _, m, n in LAYER]
    # the same finishing work, with the pre-quantisation values written out
    clip_ref = float(oracle.clip_coeff(sq, 0.05))
    assert clip_ref < 1.0
    clip_t = opt.finish_step(keys, W, prequant_outs=pres)
    clip = float(host(clip_t)[0])
    assert abs(clip - clip_ref) <= 2e-7 * clip_ref
    for (li, nm, m, n), r, g, a, (wp0, wa0), pre, w in zip(specs, ranks, gs, accs, w0, pres, W):
        _check_b200_param(oracle, opt, li, nm, m, n, r, g, a, clip, wp0, wa0, pre, w)
    opt.close()


def test_ref_full_layer_nine_parameters(oracle):
    """REF mode (two-sided, fp32, per-tensor INT8) over the nine parameters,
    fp32 weights updated in place: bit-exact against the reference's loops."""
    specs = [(3, nm, m, n) for nm, m, n in LAYER]
    opt = _opt("ref", specs, max_grad_norm=0.05)
    rng = np.random.default_rng(91)
    ws = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for _, m, n in LAYER]
    gs = [(rng.standard_normal((m, n)) * 1e-2).astype(np.float32) for _, m, n in LAYER]
    tw = [dev(w) for w in ws]
    keys = [(li, nm) for li, nm, *_ in specs]
    clip = float(host(opt.step_layer(keys, [dev(g) for g in gs], tw))[0])
    accs, pqs = [], []
    for (li, nm, m, n), g in zip(specs, gs):
        r = oracle.rank_for_param(nm, m, n)
        p = oracle.init_random_projection(m, r, li * 17)
        q = oracle.init_random_projection(n, r, li * 31)
        accs.append(oracle.project_forward(g, p, q, m, n, r).ravel())
        pqs.append((p, q, r))
    sq = sum(oracle.sqnorm_f64(a) for a in accs)
    clip_ref = float(oracle.clip_coeff(sq, 0.05))
    assert clip_ref < 1.0 and abs(clip - clip_ref) <= 2e-7 * clip_ref
    for (li, nm, m, n), w, t, a, (p, q, r) in zip(specs, ws, tw, accs, pqs):
        wd, _, m8, v8, sm, sv = oracle.galore_apply_update(a, p, q, np.zeros(r * r, np.int8), np.zeros(r * r, np.int8),
                                                           1.0, 1.0, m, n, r, clip)
        gm8, gv8, gms, gvs = opt.get_state(li, nm)
        assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8), nm
        assert host(gms)[0] == sm and host(gvs)[0] == sv, nm
        assert np.array_equal(host(t), (w - wd).astype(np.float32)), nm
    opt.close()


@pytest.mark.parametrize("m,n,r", [(256, 384, 32), (512, 256, 64)])
def test_ref_split3_small(oracle, m, n, r):
    """REF mode on the tensor cores (exact bf16 terms): accumulator and weight
    delta within 1e-6 of the reference's loops; the INT8 state, fed the GPU's
    accumulator, bit-exact."""
    specs = [(1, "d_wq", m, n, r)]
    opt = _opt("ref", specs, ref_gemm="split3")
    rng = np.random.default_rng(m + 3 * n)
    g = (rng.standard_normal((m, n)) * 1e-2).astype(np.float32)
    opt.project_and_accumulate(dev(g), 1, "d_wq")
    acc = host(opt.get_accum(1, "d_wq"))
    p = oracle.init_random_projection(m, r, 17)
    q = oracle.init_random_projection(n, r, 31)
    acc_ref = oracle.project_forward(g, p, q, m, n, r).ravel()
    assert rel_fro(acc, acc_ref) < 1e-6, rel_fro(acc, acc_ref)
    opt.apply_update(1, "d_wq", 0.7)
    delta = host(opt.take_weight_delta(1, "d_wq"))
    wd, _, m8, v8, sm, sv = oracle.galore_apply_update(acc, p, q, np.zeros(r * r, np.int8), np.zeros(r * r, np.int8),
                                                       1.0, 1.0, m, n, r, 0.7)
    gm8, gv8, gms, gvs = opt.get_state(1, "d_wq")
    assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8)
    assert host(gms)[0] == sm and host(gvs)[0] == sv
    assert rel_fro(delta, wd) < 1e-6, rel_fro(delta, wd)
    opt.close()


def test_ref_split3_c1_fp32(oracle):
    """C1's shape in REF mode (two-sided, fp32 gradient) on the tensor cores:
    the projection within 1e-5 of oracle.project_forward, the INT8 state
    bit-exact on the GPU's accumulator, and the fp32 weight after the update
    within 1e-5 of oracle.galore_apply_update's."""
    m = n = 4096
    r = 128
    opt = _opt("ref", [(0, "d_wq", m, n, r)], ref_gemm="split3")
    g = (torch.randn(m, n, generator=torch.Generator().manual_seed(1)) * 1e-3).numpy()
    w = (torch.randn(m, n, generator=torch.Generator().manual_seed(0)) * 0.02).numpy()
    tw = dev(w)
    opt.project_and_accumulate(dev(g), 0, "d_wq")
    acc = host(opt.get_accum(0, "d_wq"))
    p = oracle.init_random_projection(m, r, 0)
    q = oracle.init_random_projection(n, r, 0)
    acc_ref = oracle.project_forward(g, p, q, m, n, r).ravel()
    assert rel_fro(acc, acc_ref) < 1e-5, rel_fro(acc, acc_ref)
    sq = opt.lowrank_grad_sqnorm(0, "d_wq")
    clip = float(oracle.clip_coeff(sq, 1.0))
    opt.apply_update(0, "d_wq", clip, weight=tw)
    wd, _, m8, v8, sm, sv = oracle.galore_apply_update(acc, p, q, np.zeros(r * r, np.int8), np.zeros(r * r, np.int8),
                                                       1.0, 1.0, m, n, r, clip)
    gm8, gv8, gms, gvs = opt.get_state(0, "d_wq")
    assert np.array_equal(host(gm8), m8) and np.array_equal(host(gv8), v8)
    assert host(gms)[0] == sm and host(gvs)[0] == sv
    w_ref = (w - wd).astype(np.float32)
    assert rel_fro(host(tw) - w, w_ref - w) < 1e-5
    opt.close()
