"""tcgen05 GEMM paths: the reference-compatible fp16 projections
(galore_project.cuh:19-50) and the B200-mode one-sided projection, against
float64 references of the same (already rounded) operands."""
import numpy as np
import pytest
import torch

from tests._gpu import DEV, dev, host, ptr, rel_fro, stream

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from aethelstream_b200 import _lib
    return _lib.load()


def _h(a):
    return np.asarray(a, np.float32).astype(np.float16)


@pytest.mark.parametrize("m,n,r", [(512, 512, 16), (256, 384, 64), (1024, 2048, 128), (4096, 1024, 256),
                                   (100, 60, 12)])
def test_project_forward_fp16(oracle, lib, m, n, r):
    rng = np.random.default_rng(m + n + r)
    g = _h(rng.standard_normal((m, n)) * 1e-2)
    p = _h(oracle.init_random_projection(m, r, 17))
    q = _h(oracle.init_random_projection(n, r, 31))
    tg, tp, tq = dev(g), dev(p), dev(q)
    R = torch.empty(r, r, dtype=torch.float16, device=DEV)
    temp = torch.empty(r, n, dtype=torch.float16, device=DEV)
    assert lib.galore_project_forward(ptr(tg), ptr(tp), ptr(tq), ptr(R), ptr(temp), m, n, r, stream()) == 0
    t_ref = p.astype(np.float64).T @ g.astype(np.float64)
    # temp holds P^T G rounded to fp16 (the reference's contract), R = temp Q
    assert rel_fro(host(temp), t_ref) < 1e-3
    r_ref = host(temp).astype(np.float64) @ q.astype(np.float64)
    assert rel_fro(host(R), r_ref) < 1e-3


@pytest.mark.parametrize("m,n,r", [(512, 512, 16), (384, 256, 64), (2048, 1024, 128), (100, 60, 12)])
def test_project_backward_fp16(oracle, lib, m, n, r):
    rng = np.random.default_rng(m * 3 + r)
    nm = _h(rng.standard_normal((r, r)))
    p = _h(oracle.init_random_projection(m, r, 17))
    q = _h(oracle.init_random_projection(n, r, 31))
    out = torch.empty(m, n, dtype=torch.float16, device=DEV)
    temp = torch.empty(m, r, dtype=torch.float16, device=DEV)
    assert lib.galore_project_backward(ptr(dev(nm)), ptr(dev(p)), ptr(dev(q)), ptr(out), ptr(temp), m, n, r,
                                       stream()) == 0
    t_ref = p.astype(np.float64) @ nm.astype(np.float64)
    assert rel_fro(host(temp), t_ref) < 1e-3
    o_ref = host(temp).astype(np.float64) @ q.astype(np.float64).T
    assert rel_fro(host(out), o_ref) < 1e-3


def test_t1_roundtrip_through_gpu(oracle, lib):
    """The reference's T1 assertion (relative error < 0.1 for a rank-r G,
    test_galore_projection_roundtrip.rs:96-120) through the fp16 GPU symbols."""
    M = N = 512
    R = 16
    p32 = oracle.init_random_projection(M, R, 0xCAFEBABE - 1)
    q32 = oracle.init_random_projection(N, R, 0xB00B1E55 - 1)
    sv = (1.0 / (1.0 + np.arange(R))).astype(np.float32)
    g32 = ((p32 * sv) @ q32.T).astype(np.float32)
    tg, tp, tq = dev(_h(g32)), dev(_h(p32)), dev(_h(q32))
    Rt = torch.empty(R, R, dtype=torch.float16, device=DEV)
    tmp1 = torch.empty(R, N, dtype=torch.float16, device=DEV)
    back = torch.empty(M, N, dtype=torch.float16, device=DEV)
    tmp2 = torch.empty(M, R, dtype=torch.float16, device=DEV)
    assert lib.galore_project_forward(ptr(tg), ptr(tp), ptr(tq), ptr(Rt), ptr(tmp1), M, N, R, stream()) == 0
    assert lib.galore_project_backward(ptr(Rt), ptr(tp), ptr(tq), ptr(back), ptr(tmp2), M, N, R, stream()) == 0
    assert rel_fro(host(back), g32) < 0.1
