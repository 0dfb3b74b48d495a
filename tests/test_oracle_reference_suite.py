"""Re-run the reference crate's own test assertions on the CPU oracle.

The Rust crate cannot be compiled in this image, so the oracle's GaLore
functions are pinned by the reference test suite: galore/tests/
test_galore_projection_roundtrip.rs (T1), test_galore_quantize_roundtrip.rs
(T2) and the unit tests in quantize.rs, adamw.rs, project.rs, layer_rank.rs
and randomized_svd.rs, restated here with the same seeds and thresholds.
"""
import numpy as np
import pytest

M = N = 512
R = 16


def xorshift_uniforms(count, seed):
    """galore/tests/test_galore_projection_roundtrip.rs:21-43 (Rng, seed.max(1))."""
    s = max(seed, 1) & 0xFFFFFFFFFFFFFFFF
    out = np.empty(count, np.float32)
    mask = 0xFFFFFFFFFFFFFFFF
    for i in range(count):
        s ^= (s << 13) & mask
        s ^= s >> 7
        s ^= (s << 17) & mask
        out[i] = np.float32(s >> 40) / np.float32(1 << 24)
    return out


def random_orthonormal(oracle, rows, cols, seed):
    # Rng::new(seed) starts from `seed`; init_random_projection starts from seed + 1.
    return oracle.init_random_projection(rows, cols, seed - 1)


def lowrank_gradient(p, q, sv):
    return ((p * sv[None, :]) @ q.T).astype(np.float32)


def test_t1_projection_roundtrip_below_10_percent(oracle):
    """T1 (test_galore_projection_roundtrip.rs:96-120)."""
    p = random_orthonormal(oracle, M, R, 0xCAFEBABE)
    q = random_orthonormal(oracle, N, R, 0xB00B1E55)
    sv = (1.0 / (1.0 + np.arange(R, dtype=np.float32))).astype(np.float32)
    g = lowrank_gradient(p, q, sv)
    err = oracle.projection_roundtrip_error(g, p, q, M, N, R)
    assert err < 0.1


def test_t1_full_rank_random_bounded(oracle):
    """T1 (test_galore_projection_roundtrip.rs:122-133)."""
    p = random_orthonormal(oracle, M, R, 0xCAFEBABE)
    q = random_orthonormal(oracle, N, R, 0xB00B1E55)
    g = (xorshift_uniforms(M * N, 0x12345678) - np.float32(0.5)).reshape(M, N)
    assert oracle.projection_roundtrip_error(g, p, q, M, N, R) <= 1.0


def test_t1_fp16_path(oracle):
    """T1 (test_galore_projection_roundtrip.rs:159-190): fp16 round trip < 0.25."""
    p = random_orthonormal(oracle, M, R, 456)
    q = random_orthonormal(oracle, N, R, 789)
    sv = (1.0 / (1.0 + np.arange(R, dtype=np.float32))).astype(np.float32)
    g = lowrank_gradient(p, q, sv)
    h = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    r16 = h(oracle.project_forward(h(g), h(p), h(q), M, N, R))
    back = h(oracle.project_backward(r16, h(p), h(q), M, N, R))
    err = np.sqrt(((g.astype(np.float64) - back) ** 2).sum() / (g.astype(np.float64) ** 2).sum())
    assert err < 0.25


def t2_random_matrix(rows, cols, seed):
    """test_galore_quantize_roundtrip.rs:15-26"""
    u = xorshift_uniforms(rows * cols, seed)
    i = np.arange(rows * cols, dtype=np.float32)
    return (np.sin(i * np.float32(0.017) + u) * np.float32(0.1)).astype(np.float32)


@pytest.mark.parametrize("scale", [1e-5, 1e-3, 1e-1])
def test_t2_quantize_roundtrip(oracle, scale):
    """T2 (test_galore_quantize_roundtrip.rs:28-75): 100 low-rank AdamW steps,
    then the INT8 absmax round trip of m and v stays within 1% of max."""
    scale = np.float32(scale)
    seed = 0xDEADBEEF ^ int(np.float32(scale).view(np.uint32))
    m = n = 64
    p = t2_random_matrix(m, R, seed)
    q = t2_random_matrix(n, R, seed + 1)
    mom = np.zeros(R * R, np.float32)
    var = np.zeros(R * R, np.float32)
    for step in range(100):
        g = t2_random_matrix(m, n, seed + step + 100) * scale
        proj = oracle.project_forward(g, p, q, m, n, R).ravel()
        _, mom, var = oracle.adamw_inner_update(proj, mom, var)
    for x in (mom, var):
        qx, s = oracle.quantize_absmax(x)
        rec = oracle.dequantize_absmax(qx, s)
        rel = np.abs(x - rec).max() / np.abs(x).max()
        assert rel < 0.01


def test_unit_quantize_bounded_error(oracle):
    """quantize.rs:72-77"""
    data = (np.arange(-128, 128, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    q, s = oracle.quantize_absmax(data)
    rec = oracle.dequantize_absmax(q, s)
    assert np.abs(data - rec).max() <= oracle.absmax_scale(data) + 1e-5


def test_unit_quantize_zero_scale_is_one(oracle):
    """quantize.rs:4-13: a zero tensor has scale 1.0."""
    q, s = oracle.quantize_absmax(np.zeros(10, np.float32))
    assert s == np.float32(1.0) and not q.any()


def test_unit_round_half_away(oracle):
    """quantize.rs:21: f32::round rounds half away from zero."""
    x = np.array([127.0, 0.5, -0.5, 1.5, -2.5, 2.5], np.float32)  # scale = 1.0
    q, s = oracle.quantize_absmax(x)
    assert s == np.float32(1.0)
    assert list(q) == [127, 1, -1, 2, -3, 3]


def test_unit_lowrank_step_runs(oracle):
    """adamw.rs:208-220"""
    m = n = 8
    r = 2
    g = np.float32(0.001) * np.arange(m * n, dtype=np.float32)
    p = np.float32(0.1) * (np.arange(m * r) % 3).astype(np.float32)
    q = np.float32(0.1) * (np.arange(n * r) % 4).astype(np.float32)
    accum = oracle.project_forward(g, p, q, m, n, r)
    wd, nrm, m8, v8, sm, sv = oracle.galore_apply_update(accum, p, q, np.zeros(r * r, np.int8),
                                                         np.zeros(r * r, np.int8), 1.0, 1.0, m, n, r, 1.0)
    assert wd.size == m * n


def test_unit_adamw_inner_update_nonzero(oracle):
    """adamw.rs:222-230"""
    out, _, _ = oracle.adamw_inner_update(np.full(4, 0.1, np.float32), np.zeros(4, np.float32),
                                          np.zeros(4, np.float32))
    assert abs(out[0]) > 0.0


def test_unit_project_roundtrips(oracle):
    """project.rs:187-213"""
    g = np.arange(16, dtype=np.float32) * np.float32(0.01)
    p = (np.arange(8) % 3).astype(np.float32) * np.float32(0.1)
    q = (np.arange(8) % 5).astype(np.float32) * np.float32(0.1)
    assert oracle.projection_roundtrip_error(g, p, q, 4, 4, 2) < 1.0
    eye = np.array([1, 0, 0, 1], np.float32)
    assert oracle.projection_roundtrip_error(np.array([1, 2, 3, 4], np.float32), eye, eye, 2, 2, 2) < 1e-5


def test_unit_layer_rank(oracle):
    """layer_rank.rs:43-65"""
    assert oracle.rank_for_param("d_wq", 512, 512) == 32
    assert oracle.rank_for_param("d_wk", 512, 512) == 32
    assert oracle.rank_for_param("d_wg", 512, 512) == 16
    assert oracle.rank_for_param("d_rms1_w", 1, 512) == 1
    assert oracle.rank_for_param("d_wq", 32, 32, attn_rank=64) == 32
    assert oracle.rank_for_param("d_wg", 8, 64, attn_rank=64) == 8


def test_unit_switch_cadence(oracle):
    """randomized_svd.rs:319-324"""
    assert not oracle.should_switch(1, 200)
    assert oracle.should_switch(200, 200)
    assert oracle.should_switch(400, 200)
    assert not oracle.should_switch(200, 0)


def test_unit_clip_coeff(oracle):
    """doublepass/src/hook.rs:184-187"""
    assert oracle.clip_coeff(0.0, 1.0) == np.float32(1.0)
    assert oracle.clip_coeff(4.0, 1.0) == np.float32(1.0 / (2.0 + 1e-6))


def test_independent_restatement_of_apply_update(oracle):
    """Cross-check the C restatement of optimizer.rs:303-362 against an
    independent numpy restatement (elementwise ops in float32 round the same;
    numpy's matmul sums in another order, hence the tolerance)."""
    rng = np.random.default_rng(7)
    m, n, r = 48, 40, 8
    p = oracle.init_random_projection(m, r, 17)
    q = oracle.init_random_projection(n, r, 31)
    accum = rng.standard_normal((r, r)).astype(np.float32) * np.float32(1e-2)
    m8 = rng.integers(-127, 128, r * r).astype(np.int8)
    v8 = rng.integers(0, 128, r * r).astype(np.int8)
    sm, sv = np.float32(1e-3), np.float32(1e-6)
    clip = np.float32(0.7)
    wd, nrm, m8o, v8o, smo, svo = oracle.galore_apply_update(accum, p, q, m8, v8, sm, sv, m, n, r, float(clip))
    f = np.float32
    mom = m8.astype(f) * sm
    var = v8.astype(f) * sv
    g = accum.ravel() * clip
    mom = f(0.9) * mom + (f(1) - f(0.9)) * g
    var = f(0.999) * var + (f(1) - f(0.999)) * g * g
    nrm_np = mom / (np.sqrt(var) + f(1e-8))
    assert np.array_equal(nrm.ravel(), nrm_np)
    delta = ((p.astype(np.float64) @ nrm_np.reshape(r, r)) @ q.T.astype(np.float64)) * 1e-3
    assert np.abs(wd - delta).max() <= 1e-6 * np.abs(delta).max()
    qm, s = oracle.quantize_absmax(mom)
    assert np.array_equal(qm, m8o) and s == smo
