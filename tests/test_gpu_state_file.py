"""optimizer_states.bin from the library against the oracle's reading of the
reference layout (REF mode, version 2), and lossless save / load / continue in
B200 mode (version 3)."""
import struct

import numpy as np
import pytest
import torch

from oracle import state_file as sf
from tests._gpu import DEV, dev, host

pytestmark = pytest.mark.gpu


def _opt(mode, specs, **kw):
    from aethelstream_b200 import GaLoreConfig, GaLoreOptimizer, LayerRankConfig
    cfg = GaLoreConfig(mode=mode, layer_ranks=LayerRankConfig(), svd_refresh=False, **kw)
    return GaLoreOptimizer(cfg, specs, device=0)


def _ref_steps(opt, specs, rng, steps):
    for s in range(steps):
        for li, nm, m, n in specs:
            opt.project_and_accumulate(dev((rng.standard_normal((m, n)) * 1e-2).astype(np.float32)), li, nm)
        for li, nm, m, n in specs:
            opt.apply_update(li, nm, 1.0)
            opt.zero_accum(li, nm)
        opt.notify_step(s + 1)


def test_ref_mode_writes_the_reference_layout(oracle, tmp_path):
    specs = [(0, "d_wq", 96, 64), (1, "d_wg", 128, 96)]
    opt = _opt("ref", specs)
    _ref_steps(opt, specs, np.random.default_rng(3), 2)
    path = tmp_path / "optimizer_states.bin"
    opt.save_state(path)
    buf = path.read_bytes()
    h, layers = sf.parse(buf)
    ranks = [opt.param_info(li, nm).rank for li, nm, _, _ in specs]
    assert (h["magic"], h["version"], h["num_layers"], h["rank"], h["precision"], h["header_size"]) == \
        (sf.MAGIC, 2, 2, ranks[0], 0, 64)
    assert h["total_size"] == len(buf) and h["step_count"] == 2 and h["reserved"] == bytes(12)
    assert (h["beta1"], h["beta2"], h["eps"]) == (np.float32(0.9), np.float32(0.999), np.float32(1e-8))
    descs = sf.build_descriptors([(m, n) for *_, m, n in specs], ranks)
    for (li, nm, m, n), L, d in zip(specs, layers, descs):
        assert (L["m"], L["n"], L["rank"], L["offset"]) == d
        P, Q = opt.get_projector(li, nm)
        assert np.array_equal(L["p_bits"].ravel(), oracle.galore_f32_to_f16(host(P)))
        assert np.array_equal(L["q_bits"].ravel(), oracle.galore_f32_to_f16(host(Q)))
        m8, v8, ms, vs = [host(x) for x in opt.get_state(li, nm)]
        assert np.array_equal(L["m8"], m8) and np.array_equal(L["v8"], v8)
        assert L["scale_m"] == ms[0] and L["scale_v"] == vs[0]

    # GaLoreOptimizer::open semantics: projectors read back through f16, state as stored
    fresh = _opt("ref", specs)
    fresh.load_state(path)
    assert fresh.step_count() == 2
    for (li, nm, m, n), L in zip(specs, layers):
        P, Q = fresh.get_projector(li, nm)
        assert np.array_equal(host(P).ravel(), oracle.galore_f16_to_f32(L["p_bits"].ravel()))
        assert np.array_equal(host(Q).ravel(), oracle.galore_f16_to_f32(L["q_bits"].ravel()))
        m8, v8, ms, vs = [host(x) for x in fresh.get_state(li, nm)]
        assert np.array_equal(m8, L["m8"]) and ms[0] == L["scale_m"]
        assert not host(fresh.get_accum(li, nm)).any()
    opt.close()
    fresh.close()


def test_b200_mode_save_load_continue_is_lossless(tmp_path):
    from aethelstream_b200 import nf4_quantize
    specs = [(0, "d_wq", 512, 256, 64), (0, "d_wd", 256, 768, 64)]
    rng = np.random.default_rng(8)
    a = _opt("b200", specs, state_codec="dynamic")
    ws = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for _, _, m, n, _ in specs]
    grads = [[(rng.standard_normal((m, n)) * 1e-3).astype(np.float32) for _, _, m, n, _ in specs] for _ in range(3)]
    keys = [(li, nm) for li, nm, *_ in specs]
    Wa = [nf4_quantize(dev(w)) for w in ws]
    for s in range(2):
        a.step_layer(keys, [dev(g).to(torch.bfloat16) for g in grads[s]], Wa)
        a.notify_step(s + 1)
    path = tmp_path / "state_v3.bin"
    a.save_state(path)
    assert struct.unpack_from("<II", path.read_bytes(), 0) == (sf.MAGIC, 3)
    b = _opt("b200", specs, state_codec="dynamic")
    b.load_state(path)
    assert b.step_count() == 2
    for li, nm, *_ in specs:
        for x, y in zip(a.get_state(li, nm), b.get_state(li, nm)):
            assert np.array_equal(host(x), host(y))
        pa, qa = a.get_projector(li, nm)
        pb, qb = b.get_projector(li, nm)
        assert np.array_equal(host(pa if pa is not None else qa), host(pb if pb is not None else qb))
    # the same third step on both gives identical weights and state
    Wb = [type(w)(w.packed.clone(), w.absmax.clone(), w.shape) for w in Wa]
    ca = a.step_layer(keys, [dev(g).to(torch.bfloat16) for g in grads[2]], Wa)
    cb = b.step_layer(keys, [dev(g).to(torch.bfloat16) for g in grads[2]], Wb)
    assert host(ca)[0] == host(cb)[0]
    for wa, wb in zip(Wa, Wb):
        assert torch.equal(wa.packed, wb.packed) and torch.equal(wa.absmax, wb.absmax)
    for li, nm, *_ in specs:
        for x, y in zip(a.get_state(li, nm), b.get_state(li, nm)):
            assert np.array_equal(host(x), host(y))
    a.close()
    b.close()


def test_load_errors(tmp_path):
    from aethelstream_b200 import AethError, _lib
    specs = [(0, "d_wq", 96, 64)]
    opt = _opt("ref", specs)
    path = tmp_path / "s.bin"
    opt.save_state(path)
    other = _opt("ref", [(0, "d_wq", 128, 64)])
    with pytest.raises(AethError) as e:
        other.load_state(path)
    assert e.value.status == _lib.AETH_ERR_SHAPE
    with pytest.raises(AethError) as e:
        opt.load_state(tmp_path / "missing.bin")
    assert e.value.status == _lib.AETH_ERR_NOT_FOUND
    bad = bytearray(path.read_bytes())
    bad[0] ^= 0xFF
    (tmp_path / "bad.bin").write_bytes(bytes(bad))
    with pytest.raises(AethError) as e:
        opt.load_state(tmp_path / "bad.bin")
    assert e.value.status == _lib.AETH_ERR_CONFIG
    b200 = _opt("b200", [(0, "d_wq", 128, 64, 16)])
    with pytest.raises(AethError) as e:
        b200.load_state(path)  # a version 2 file in B200 mode
    assert e.value.status == _lib.AETH_ERR_CONFIG
    opt.close()
    other.close()
    b200.close()
