"""The streamed-weight decode and BF16 write-back restatements (oracle) against
the reference's own tests, re-run on them:

* flowcast/tests/test_quantized_stream.rs:29-72 (T8-1..T8-4: INT8 and NF4 decode
  error bounds and output sizes) and the f32 -> f16 conversion of
  flowcast/src/decode.rs:191-210 against a line-by-line transcription;
* doublepass/tests/test_stochastic_rounding.rs (expectation within one ULP,
  loss decrease against fp32, sub-ULP steps beating truncation, determinism,
  exact round trip) and the LCG of doublepass/src/precision.rs:212-217 against
  a Python transcription.
"""
import struct

import numpy as np


def _bits(x):
    return struct.unpack("<I", struct.pack("<f", np.float32(x)))[0]


def _f16_to_f32(bits):
    """test_quantized_stream.rs:15-27 (the test's own decoder, including its 2^-24 subnormal scale)."""
    sign = -1.0 if (bits >> 15) & 1 else 1.0
    exp = (bits >> 10) & 0x1F
    mant = bits & 0x3FF
    if exp == 0:
        return sign * mant / 16777216.0
    if exp == 31:
        return sign * float("inf")
    return sign * (1.0 + mant / 1024.0) * 2.0 ** (exp - 15)


def _fc_f32_to_f16_py(v):
    """decode.rs:191-210, transcribed."""
    bits = _bits(v)
    sign = bits >> 31
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp == 0xFF:
        return (sign << 15) | 0x7C00 | (0x0200 if mant else 0)
    e16 = exp - 127 + 15
    if e16 <= 0:
        return sign << 15
    if e16 >= 31:
        return (sign << 15) | 0x7C00
    return (sign << 15) | (e16 << 10) | (mant >> 13)


def test_f32_to_f16_matches_transcription(oracle):
    rng = np.random.default_rng(3)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 4000),
        np.array([0.0, -0.0, 65504.0, 65520.0, 1e30, -1e30, 6.1e-5, 5.9e-5, np.inf, -np.inf, np.nan], np.float32),
    ]).astype(np.float32)
    for v in vals:
        assert oracle.fc_f32_to_f16(v) == _fc_f32_to_f16_py(v), v


def test_int8_decode_error_within_bound_and_shape(oracle):
    """test_quantized_stream.rs:29-52 (T8-1/T8-3)."""
    max_abs = np.float32(127.0)
    scale = np.float32(max_abs / np.float32(127.0))
    src = np.arange(0, 128, dtype=np.uint8).view(np.int8)
    out = oracle.fc_decode_int8(src, [scale], 1)
    assert out.size == src.size  # two bytes per element
    for raw, h in zip(src, out):
        expected = float(np.float32(raw) * scale)
        assert abs(_f16_to_f32(int(h)) - expected) <= max_abs / 127.0 + 1e-3


def test_int8_decode_channels_and_missing_scales(oracle):
    """decode.rs:63-86: channel = i / (n / num_channels); a channel past the
    scale list decodes with 1.0."""
    src = np.array([1, -2, 3, -4, 5, -6, 7], np.int8)
    out = oracle.fc_decode_int8(src, [0.5, 2.0], 2)  # 3 elements per channel, element 6 is channel 2
    want = [oracle.fc_f32_to_f16(np.float32(v) * np.float32(s))
            for v, s in zip(src, [0.5] * 3 + [2.0] * 3 + [1.0])]
    assert list(out) == want
    assert list(oracle.fc_decode_int8(src, [3.0], 0)) == [oracle.fc_f32_to_f16(np.float32(v) * 3) for v in src]


def test_int4_decode_tolerance_shape_and_nibble_order(oracle):
    """test_quantized_stream.rs:54-72 (T8-2/T8-4), and the low-nibble-first
    order of decode.rs:95-97 (shard_engine packs the high nibble first)."""
    src = np.array([(i << 4) | i for i in range(8)], np.uint8)
    out = oracle.fc_decode_int4(src, 1.0)
    assert out.size == 2 * src.size
    assert all(abs(_f16_to_f32(int(h))) <= 1.0 + 0.3 for h in out)
    out = oracle.fc_decode_int4(np.array([0x7F], np.uint8), 2.0)  # low nibble 0xF first: +1.0, then code 7: 0.0
    assert _f16_to_f32(int(out[0])) == 2.0 and _f16_to_f32(int(out[1])) == 0.0


def _lcg_py(state):
    state = (state * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
    return (state >> 33) & 0xFFFF, state


def test_lcg_matches_transcription(oracle):
    s_c = s_py = 0xDEAD_BEEF_1234_5678
    for _ in range(1000):
        r_c, s_c = oracle.lcg_next(s_c)
        r_py, s_py = _lcg_py(s_py)
        assert (r_c, s_c) == (r_py, s_py)


def _bf16_to_f32(b):
    return struct.unpack("<f", struct.pack("<I", b << 16))[0]


def test_stochastic_round_expectation(oracle):
    """test_stochastic_rounding.rs:49-80: E[SR(x)] = x within one bf16 ULP."""
    for val in [1.0, -0.5, 3.14159, 0.001, 100.0, -7.5]:
        v = np.float32(val)
        total = sum(_bf16_to_f32(oracle.stochastic_round_to_bf16(v, r)) for r in range(0, 65536, 16)) / 4096.0
        trunc = _bf16_to_f32(_bits(v) >> 16)
        e = (_bits(abs(trunc)) >> 23) & 0xFF
        ulp = struct.unpack("<f", struct.pack("<I", max(e - 7, 0) << 23))[0] if e > 0 else np.finfo(np.float32).tiny
        assert abs(total - val) <= ulp + np.finfo(np.float32).eps * abs(val)


def test_sr_update_loss_decreases_like_fp32(oracle):
    """test_stochastic_rounding.rs:86-128."""
    n, lr, steps = 64, np.float32(0.05), 300
    target = (np.arange(n, dtype=np.float32) * np.float32(0.1) - np.float32(3.0)).astype(np.float32)
    w = np.zeros(n, np.float32)
    init = float(np.sum((w - target) ** 2 * 0.5))
    rng = 0xDEAD_BEEF_1234_5678
    for _ in range(steps):
        delta = (-lr * (w - target)).astype(np.float32)
        w, rng = oracle.apply_galore_bf16_update(w, delta, rng)
    assert float(np.sum((w - target) ** 2 * 0.5)) < init * 0.05


def test_sr_beats_truncation_for_sub_ulp_steps(oracle):
    """test_stochastic_rounding.rs:145-189."""
    n, lr, steps = 64, np.float32(0.01), 1000
    target = np.full(n, 192.0, np.float32)
    w_det = np.full(n, 128.0, np.float32)
    for _ in range(steps):
        d = (-lr * (w_det - target)).astype(np.float32)
        w_det = ((w_det + d).astype(np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    w_sr = np.full(n, 128.0, np.float32)
    rng = 0xFEED_FACE_CAFE_1234
    for _ in range(steps):
        w_sr, rng = oracle.apply_galore_bf16_update(w_sr, (-lr * (w_sr - target)).astype(np.float32), rng)
    loss = lambda w: float(np.sum((w - target) ** 2 * 0.5))  # noqa: E731
    init = loss(np.full(n, 128.0, np.float32))
    assert loss(w_det) > init * 0.99
    assert loss(w_sr) < loss(w_det) * 0.5 and loss(w_sr) < init * 0.01


def test_sr_update_deterministic_and_round_trip(oracle):
    """test_stochastic_rounding.rs:209-251."""
    n = 32
    delta = (-(np.arange(n, dtype=np.float32)) * np.float32(0.01)).astype(np.float32)
    w1, s1 = oracle.apply_galore_bf16_update(np.ones(n, np.float32), delta, 0x1111_2222_3333_4444)
    w2, s2 = oracle.apply_galore_bf16_update(np.ones(n, np.float32), delta, 0x1111_2222_3333_4444)
    assert np.array_equal(w1.view(np.uint32), w2.view(np.uint32)) and s1 == s2
    for v in [0.0, 1.0, 2.0, 0.5, -1.0, 128.0, 0.00390625]:
        b = _bits(v)
        assert _bits(_bf16_to_f32(b >> 16)) == b
        assert oracle.stochastic_round_to_bf16(v, 0) == b >> 16  # nothing to round up


def test_sr_saturates_at_all_ones(oracle):
    """precision.rs:130-133: saturating_add keeps 0xFFFF (a NaN pattern) from wrapping to +0."""
    nan_ones = struct.unpack("<f", struct.pack("<I", 0xFFFFFFFF))[0]
    assert oracle.stochastic_round_to_bf16(nan_ones, 0) == 0xFFFF
