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


def test_sketch_entry_equals_the_seeded_draw(oracle):
    """ref_randomized_svd_sketch from the drawn sketch is ref_randomized_svd."""
    rng = np.random.default_rng(4)
    m, n, r, p = 96, 80, 8, 6
    g = rng.standard_normal((m, n)).astype(np.float32)
    seed = oracle.rsvd_seed(7)
    omega = oracle.rsvd_omega(seed, n * (r + p)).reshape(n, r + p)
    a = oracle.randomized_svd(g, m, n, r, p, seed)
    b = oracle.randomized_svd(g, m, n, r, p, 0, omega=omega)
    assert a[0] == b[0] == 0
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


def _f64_projections(g, omega, r):
    """The same algorithm in f64 (numpy), with the reference's Gram-Schmidt
    and its 50-rotation Jacobi."""
    def mgs(q, clamp):
        q = q.copy()
        for j in range(q.shape[1]):
            for i in range(j):
                q[:, j] -= (q[:, i] @ q[:, j]) * q[:, i]
            s = q[:, j] @ q[:, j]
            q[:, j] /= math.sqrt(max(s, 1e-12) if clamp else s)
        return q

    def jacobi(a):
        a = a.copy()
        n = a.shape[0]
        u = np.eye(n)
        for _ in range(50):
            t = np.abs(np.triu(a, 1))
            p, q = divmod(int(np.argmax(t)), n)
            if t[p, q] < 1e-10:
                break
            tau = (a[q, q] - a[p, p]) / (2 * a[p, q])
            t_ = 1 / (tau + math.sqrt(1 + tau * tau)) if tau >= 0 else -1 / (-tau + math.sqrt(1 + tau * tau))
            c = 1 / math.sqrt(1 + t_ * t_)
            s = t_ * c
            for k in range(n):
                akp, akq = a[k, p], a[k, q]
                a[k, p] = c * akp - s * akq
                a[p, k] = a[k, p]
                a[k, q] = s * akp + c * akq
                a[q, k] = a[k, q]
            a[p, q] = a[q, p] = 0.0
            up, uq = u[:, p].copy(), u[:, q].copy()
            u[:, p], u[:, q] = c * up - s * uq, s * up + c * uq
        return u

    g, omega = g.astype(np.float64), omega.astype(np.float64)
    y = mgs(g @ omega, False)
    b = y.T @ g
    u = jacobi(b @ b.T)
    return y @ u[:, :r], mgs(b.T @ u[:, :r], True)


def test_f32_reference_is_close_to_its_f64_restatement(oracle):
    """At these shapes the reference's f32 loops land within 1e-5 of the same
    algorithm in f64: a device refresh within 1e-5 of the oracle is within
    the reference's own rounding."""
    rng = np.random.default_rng(20)
    m, n, r, p = 256, 384, 16, 8
    k = r + p + 8
    g = ((rng.standard_normal((m, k)) * np.geomspace(1.0, 0.05, k)) @ rng.standard_normal((k, n))
         + 0.01 * rng.standard_normal((m, n))).astype(np.float32)
    omega = oracle.rsvd_omega(oracle.rsvd_seed(200), n * (r + p)).reshape(n, r + p)
    st, p32, q32 = oracle.randomized_svd(g, m, n, r, p, 0, omega=omega)
    p64, q64 = _f64_projections(g, omega, r)
    assert st == 0
    assert np.linalg.norm(p32 - p64) / np.linalg.norm(p64) < 1e-5
    assert np.linalg.norm(q32 - q64) / np.linalg.norm(q64) < 1e-5
