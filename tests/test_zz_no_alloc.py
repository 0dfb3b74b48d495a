"""galore_project_forward_noalloc against galore_project_forward.

The allocation-free entry point serves callers that cannot allocate device
memory where they call the projection (for example a hook running inside
another framework's step, whose device memory that framework's caching
allocator already holds).  It keeps the P^T G intermediate in a fixed array
inside the library instead of a caller-provided temp buffer.  This file is
named so that pytest collects it after every other test; it must pass both on
its own in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from tests._gpu import DEV, dev, host, ptr, rel_fro, stream

pytestmark = pytest.mark.gpu

MAX_ELEMS = 8 * 1024 * 1024  # r * n limit of the fixed intermediate


@pytest.fixture(scope="module")
def lib():
    from aethelstream_b200 import _lib
    return _lib.load()


def _inputs(m, n, r, seed):
    rng = np.random.default_rng(seed)
    g = (rng.standard_normal((m, n)) * 1e-2).astype(np.float16)
    p = (rng.standard_normal((m, r)) / np.sqrt(m)).astype(np.float16)
    q = (rng.standard_normal((n, r)) / np.sqrt(n)).astype(np.float16)
    return dev(g), dev(p), dev(q)


def test_noalloc_matches_forward_on_consecutive_calls(lib):
    # The second and third calls use smaller r * n than the first, so the shared
    # array still holds data from an earlier call beyond what they write.
    for call, (m, n, r, seed) in enumerate([(1024, 2048, 128, 11), (512, 768, 64, 12), (512, 768, 64, 13)]):
        tg, tp, tq = _inputs(m, n, r, seed)
        r_ref = torch.empty(r, r, dtype=torch.float16, device=DEV)
        temp = torch.empty(r, n, dtype=torch.float16, device=DEV)
        assert lib.galore_project_forward(ptr(tg), ptr(tp), ptr(tq), ptr(r_ref), ptr(temp), m, n, r, stream()) == 0
        r_na = torch.full((r, r), float("nan"), dtype=torch.float16, device=DEV)
        assert lib.galore_project_forward_noalloc(ptr(tg), ptr(tp), ptr(tq), ptr(r_na), m, n, r, stream()) == 0, call
        got, want = host(r_na), host(r_ref)
        assert np.isfinite(got).all(), call
        assert rel_fro(got, want) < 1e-3, call
        # and against the float64 product of the same fp16 operands
        exact = (host(tp).astype(np.float64).T @ host(tg).astype(np.float64)) @ host(tq).astype(np.float64)
        assert rel_fro(got, exact) < 2e-3, call


def test_noalloc_rejects_sizes_beyond_the_fixed_array(lib):
    small = torch.zeros(16, dtype=torch.float16, device=DEV)
    # r * n = 128 * 65537 > 8,388,608: refused before any device work
    st = lib.galore_project_forward_noalloc(ptr(small), ptr(small), ptr(small), ptr(small), 64, 65537, 128, stream())
    assert st == -4  # AETH_ERR_UNSUPPORTED
    assert lib.aeth_last_error() == -4
    assert lib.galore_project_forward_noalloc(None, None, None, None, 64, 64, 16, stream()) == -1
    assert lib.galore_project_forward_noalloc(ptr(small), ptr(small), ptr(small), ptr(small), 0, 64, 16,
                                              stream()) == -1
