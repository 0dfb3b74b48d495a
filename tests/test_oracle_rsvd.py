"""CPU oracle of the randomized-SVD subspace refresh (galore/src/randomized_svd.rs).

The reference ships no golden vectors for this path (its Rust crate cannot
be built here), so the C restatement is pinned by the reference's own unit
tests (randomized_svd.rs:304-325) and by independent pure-Python
transcriptions of its generator and its Jacobi loop on small inputs.
"""
import math

import numpy as np
import pytest

f32 = np.float32


def _xorshift(s):
    s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
    s ^= s >> 7
    s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
    return s


def test_reference_unit_test_shapes(oracle):
    # randomized_svd.rs:304-317
    m = n = 32
    g = np.array([((i * 7) % 11) * 0.01 for i in range(m * n)], np.float32).reshape(m, n)
    st, p, q = oracle.randomized_svd(g, m, n, 4, 4, 42)
    assert st == 0 and p.shape == (m, 4) and q.shape == (n, 4)


def test_switch_cadence(oracle):
    # randomized_svd.rs:319-324
    assert not oracle.should_switch(1, 200)
    assert oracle.should_switch(200, 200) and oracle.should_switch(400, 200)
    assert not oracle.should_switch(0, 200) and not oracle.should_switch(5, 0)


def test_omega_matches_a_python_transcription(oracle):
    # Rng (randomized_svd.rs:38-66), evaluated in f32 step by step
    seed = oracle.rsvd_seed(3)
    got = oracle.rsvd_omega(seed, 64)
    s = max(seed, 1)
    for i in range(64):
        s = _xorshift(s)
        u1 = max(f32(s >> 40) / f32(1 << 24), f32(1e-7))
        s = _xorshift(s)
        u2 = f32(s >> 40) / f32(1 << 24)
        two_pi = f32(2.0) * f32(math.pi)
        # libm logf / cosf are within an ulp of the f64 values rounded to f32
        want = f32(math.sqrt(f32(-2.0) * f32(math.log(u1)))) * f32(math.cos(f32(two_pi * u2)))
        assert abs(float(got[i]) - float(want)) <= 4e-7 * max(1.0, abs(float(want))), i


def test_omega_is_standard_normal(oracle):
    x = oracle.rsvd_omega(oracle.rsvd_seed(1), 200_000).astype(np.float64)
    assert abs(x.mean()) < 0.01 and abs(x.var() - 1.0) < 0.02


def _jacobi_py(a):
    """jacobi_eigenvectors transcribed loop for loop in numpy f32 scalars."""
    a = a.astype(np.float32).copy()
    n = a.shape[0]
    u = np.eye(n, dtype=np.float32)
    for _ in range(50):
        max_off, p, q = f32(0), 0, 1
        for i in range(n):
            for j in range(i + 1, n):
                v = abs(a[i, j])
                if v > max_off:
                    max_off, p, q = v, i, j
        if max_off < f32(1e-10):
            break
        app, aqq, apq = a[p, p], a[q, q], a[p, q]
        tau = (aqq - app) / (f32(2) * apq)
        root = np.sqrt(f32(1) + tau * tau)
        t = f32(1) / (tau + root) if tau >= 0 else f32(-1) / (-tau + root)
        c = f32(1) / np.sqrt(f32(1) + t * t)
        s = t * c
        for k in range(n):
            mkp, mkq = a[k, p], a[k, q]
            a[k, p] = c * mkp - s * mkq
            a[p, k] = a[k, p]
            a[k, q] = s * mkp + c * mkq
            a[q, k] = a[k, q]
        a[p, q] = a[q, p] = f32(0)
        for k in range(n):
            ukp, ukq = u[k, p], u[k, q]
            u[k, p] = c * ukp - s * ukq
            u[k, q] = s * ukp + c * ukq
    return u, a


@pytest.mark.parametrize("n", [2, 5, 9])
def test_jacobi_matches_the_transcribed_loop(oracle, n):
    rng = np.random.default_rng(n)
    b = rng.standard_normal((n, n + 3)).astype(np.float32)
    a = (b @ b.T).astype(np.float32)
    u, m = oracle.rsvd_jacobi(a)
    u_py, m_py = _jacobi_py(a)
    assert np.array_equal(u, u_py) and np.array_equal(m, m_py)


def test_projections_are_orthonormal_and_capture_the_range(oracle):
    rng = np.random.default_rng(5)
    m, n, r = 96, 160, 8
    # rank-r signal plus small noise: the refresh must find its column space
    a = rng.standard_normal((m, r)).astype(np.float32)
    b = rng.standard_normal((r, n)).astype(np.float32)
    g = (a @ b + 1e-3 * rng.standard_normal((m, n))).astype(np.float32)
    st, p, q = oracle.randomized_svd(g, m, n, r, 4, oracle.rsvd_seed(1))
    assert st == 0
    assert np.abs(p.T @ p - np.eye(r)).max() < 1e-4
    assert np.abs(q.T @ q - np.eye(r)).max() < 1e-4
    # P spans a subspace of range(Q^) that holds most of G
    captured = np.linalg.norm(p.T @ g) / np.linalg.norm(g)
    assert captured > 0.3


def test_errors(oracle):
    g = np.ones((16, 16), np.float32)
    assert oracle.randomized_svd(g, 16, 16, 0, 4, 1)[0] == -2    # rank 0: GaLoreError::Config
    assert oracle.randomized_svd(g, 16, 16, 10, 8, 1)[0] == -2   # r + p > min(m, n)
    assert oracle.randomized_svd(np.zeros((16, 16), np.float32), 16, 16, 2, 2, 1)[0] == -3  # Linalg
