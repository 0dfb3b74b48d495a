"""The B200-mode extensions of the oracle (parity unpinned by the reference):
checked for reduction to the reference definitions where one exists, and for
their own algebraic properties otherwise."""
import numpy as np
import pytest


def test_block_linear_reduces_to_per_tensor(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(5000).astype(np.float32) * np.float32(1e-3)
    q_ref, s_ref = oracle.quantize_absmax(x)
    q, s = oracle.block_quantize(x, block=8192, codec=oracle.CODEC_LINEAR)
    assert np.array_equal(q, q_ref) and s[0] == s_ref


def test_block_linear_is_per_block(oracle):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(3 * 2048 + 100).astype(np.float32)
    q, s = oracle.block_quantize(x, block=2048, codec=oracle.CODEC_LINEAR)
    assert s.size == 4
    for b in range(4):
        qb, sb = oracle.quantize_absmax(x[b * 2048:(b + 1) * 2048])
        assert np.array_equal(q[b * 2048:(b + 1) * 2048], qb) and s[b] == sb


@pytest.mark.parametrize("signed", [True, False])
def test_dynamic_codec_roundtrip(oracle, signed):
    rng = np.random.default_rng(2)
    x = rng.standard_normal(4096).astype(np.float32)
    x = x if signed else np.abs(x)
    q, s = oracle.block_quantize(x, block=2048, codec=oracle.CODEC_DYNAMIC, signed=signed)
    rec = oracle.block_dequantize(q, s, block=2048, codec=oracle.CODEC_DYNAMIC, signed=signed)
    m = oracle.dynamic_map(signed)
    # worst case: half the widest gap, or -1 mapped to the most negative entry
    bound = max(0.5 * float(np.diff(m).max()), 1.0 + float(m[0]) if signed else 0.0)
    for b in range(2):
        blk = slice(b * 2048, (b + 1) * 2048)
        assert np.abs(x[blk] - rec[blk]).max() <= bound * s[b] * (1 + 1e-5)
    # nearest-entry property
    xn = x[:2048] * (np.float32(1.0) / s[0])
    d = np.abs(xn[:, None] - m[None, :])
    assert np.array_equal(q[:2048].view(np.uint8), d.argmin(axis=1).astype(np.uint8))


def test_adam_state_reduces_to_reference(oracle):
    """b2_adam_state with the linear codec and one block over the state is the
    reference's apply_update state transition (adamw.rs:79-135)."""
    rng = np.random.default_rng(3)
    r = 16
    accum = rng.standard_normal(r * r).astype(np.float32) * np.float32(1e-2)
    m8 = rng.integers(-127, 128, r * r).astype(np.int8)
    v8 = rng.integers(0, 128, r * r).astype(np.int8)
    sm, sv = np.float32(2e-3), np.float32(3e-6)
    clip = 0.5
    p = oracle.init_random_projection(r, r, 17)
    _, nrm, m8r, v8r, smr, svr = oracle.galore_apply_update(accum, p, p, m8, v8, sm, sv, r, r, r, clip)
    nb, m8b, v8b, smb, svb = oracle.b2_adam_state(accum, m8, v8, [sm], [sv], 4096, oracle.CODEC_LINEAR, clip)
    assert np.array_equal(m8b, m8r) and np.array_equal(v8b, v8r)
    assert smb[0] == smr and svb[0] == svr
    assert np.array_equal(nb, oracle.bf16_round(nrm.ravel()))


@pytest.mark.parametrize("m,n", [(96, 64), (64, 96), (64, 64)])
def test_one_sided_projection(oracle, m, n):
    rng = np.random.default_rng(4)
    r = 8
    g = rng.standard_normal((m, n)).astype(np.float32)
    right = oracle.side_is_right(m, n)
    s = n if right else m
    proj = oracle.init_random_projection(s, r, 31)
    racc = np.zeros(max(m, n) * r, np.float32)
    out = oracle.b2_project_accumulate(g, proj, racc, m, n, r).reshape(max(m, n), r)
    expect = (g.astype(np.float64) @ proj) if right else (g.T.astype(np.float64) @ proj)
    assert np.abs(out - expect).max() < 1e-5
    assert right == (m >= n)


def test_apply_weight_zero_update_is_idempotent(oracle):
    """NF4 requantisation of an unchanged dequantised block reproduces it."""
    rng = np.random.default_rng(5)
    m, n, r = 64, 128, 8
    w = rng.standard_normal(m * n).astype(np.float32) * np.float32(0.02)
    wp, wa = oracle.nf4_quantize(w)
    nz = np.zeros(n * r, np.float32)
    proj = oracle.init_random_projection(m, r, 1)
    wp2, wa2, pre, dw = oracle.b2_apply_weight(nz, proj, m, n, r, wp, wa, 1e-3)
    assert np.array_equal(wp2, wp) and np.array_equal(wa2, wa)


def test_apply_weight_formula(oracle):
    rng = np.random.default_rng(6)
    m, n, r = 128, 64, 16
    w = rng.standard_normal(m * n).astype(np.float32) * np.float32(0.02)
    wp, wa = oracle.nf4_quantize(w)
    nb = oracle.bf16_round(rng.standard_normal(m * r).astype(np.float32))
    proj = oracle.bf16_round(oracle.init_random_projection(n, r, 2))
    lr = np.float32(1e-3)
    wp2, wa2, pre, dw = oracle.b2_apply_weight(nb, proj, m, n, r, wp, wa, float(lr))
    d = (nb.reshape(m, r).astype(np.float64) @ proj.reshape(n, r).T.astype(np.float64)).astype(np.float32)
    w0 = oracle.nf4_dequant_f32(wp, wa, m * n)
    expect = w0 - (lr * d.ravel()).astype(np.float32)
    assert np.array_equal(pre, expect)
    p3, a3 = oracle.nf4_requant(pre)
    assert np.array_equal(p3, wp2) and np.array_equal(a3, wa2)


def test_lomo_beta0_is_clipped_sgd(oracle):
    """With beta = 0 the LOMO step is w -= lr * clip * g (doublepass/tests/test_resume.rs:138-152)."""
    rng = np.random.default_rng(7)
    n = 4096
    g = oracle.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32) * np.float32(1e-3))
    w = rng.standard_normal(n).astype(np.float32) * np.float32(0.02)
    wp, wa = oracle.nf4_quantize(w)
    sq = oracle.lomo_sqnorm(g)
    assert abs(sq - float((oracle.bf16_bits_to_f32(g).astype(np.float64) ** 2).sum())) < 1e-12 * sq
    clip = oracle.clip_coeff(sq, 1.0)
    mom8 = np.zeros(n, np.int8)
    ms = np.ones(n // 2048, np.float32)
    _, _, _, _, pre = oracle.lomo_update(g, float(clip), 0.0, 1e-3, 2048, oracle.CODEC_LINEAR, mom8, ms, wp, wa)
    gs = oracle.bf16_bits_to_f32(g) * clip
    expect = oracle.nf4_dequant_f32(wp, wa, n) - (np.float32(1e-3) * gs).astype(np.float32)
    assert np.array_equal(pre, expect)
