"""The 8-bit dynamic map of the blockwise INT8 state (AETH_CODEC_BLOCK_DYNAMIC),
compared entry by entry with two restatements of its published construction
(Dettmers et al. 2021, dynamic tree quantisation: an optional sign bit, E
leading zero bits selecting the decade 10^-E, an indicator bit, and the
remaining bits as the midpoints of equal bins over [0.1, 1]; plus 0 and 1):

* exact rational arithmetic rounded once to fp32 -- the library's map is the
  correctly rounded one, entry for entry;
* the fp32 tensor arithmetic the published implementation uses (linspace of
  the bin edges, midpoints and the decade factor, all fp32), restated here
  with torch -- it rounds several times, so some entries land one or two
  ulp away; the test bounds that difference and counts it.

No reference pin exists for this map: the reference's INT8 state is
per-tensor linear (galore/src/quantize.rs:4-34)."""
from fractions import Fraction

import numpy as np
import pytest


def _library_map(signed):
    import ctypes as C

    from aethelstream_b200 import _lib as L
    out = (C.c_float * 256)()
    L.check(L.load().aeth_dynamic_map(1 if signed else 0, out), "aeth_dynamic_map")
    return np.array(out[:], np.float32)


def _levels(signed):
    # fraction bits after the sign (signed only), the E zero bits and the indicator
    return [(e, 2 ** ((6 if signed else 7) - e)) for e in range(7)]


def _exact_map(signed):
    vals = [Fraction(0), Fraction(1)]
    for e, lv in _levels(signed):
        for j in range(lv):
            v = Fraction(1, 10 ** e) * (Fraction(1, 10) + Fraction(9, 10) * Fraction(2 * j + 1, 2 * lv))
            vals.append(v)
            if signed:
                vals.append(-v)
    assert len(vals) == 256
    return np.sort(np.array([np.float32(float(v)) for v in vals], np.float32))


def _fp32_tensor_map(signed):
    import torch
    vals = [0.0, 1.0]
    for e, lv in _levels(signed):
        edges = torch.linspace(0.1, 1.0, lv + 1, dtype=torch.float32)
        mids = (edges[:-1] + edges[1:]) / 2.0
        scaled = mids * (10.0 ** -e)
        vals += scaled.tolist()
        if signed:
            vals += (-scaled).tolist()
    assert len(vals) == 256
    return np.sort(np.array(vals, np.float32))


@pytest.mark.parametrize("signed", [True, False])
def test_dynamic_map_is_correctly_rounded(signed):
    assert np.array_equal(_library_map(signed), _exact_map(signed))


@pytest.mark.parametrize("signed", [True, False])
def test_dynamic_map_against_fp32_tensor_construction(signed):
    mine = _library_map(signed)
    pub = _fp32_tensor_map(signed)
    assert np.array_equal(np.sign(mine), np.sign(pub))
    ulp = np.abs(mine.view(np.int32).astype(np.int64) - pub.view(np.int32).astype(np.int64))
    assert ulp.max() <= 2, ulp.max()
    rel = np.abs(mine.astype(np.float64) - pub) / np.maximum(np.abs(pub.astype(np.float64)), 1e-30)
    assert rel.max() < 2.5e-7
    # the fp32 construction rounds the bin edges and the midpoints separately:
    # a minority of the entries move, none by more than the bound above
    assert (ulp > 0).sum() < 128


@pytest.mark.parametrize("signed", [True, False])
def test_dynamic_map_oracle_agrees(oracle, signed):
    assert np.array_equal(np.asarray(oracle.dynamic_map(signed), np.float32), _library_map(signed))
