"""CPU restatement of optimizer_states.bin version 2 and of galore's half
conversion, pinned by the reference's own unit tests (state_file.rs:595-657)
and by a pure-Python transcription of project.rs:137-184."""
import math
import struct

import numpy as np
import pytest

from oracle import state_file as sf


def _f32_to_f16_py(x):
    """project.rs:137-158, transcribed line by line."""
    bits = struct.unpack("<I", struct.pack("<f", x))[0]
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    frac = bits & 0x7FFFFF
    if exp == 0xFF:
        return sign | 0x7C00 | ((frac >> 13) & 0x3FF)
    new_exp = exp - 127 + 15
    if new_exp >= 0x1F:
        return sign | 0x7C00
    if new_exp <= 0:
        if new_exp < -10:
            return sign
        mant = (frac | 0x800000) >> (1 - new_exp)
        return (sign | ((mant + 0x1000) >> 13)) & 0xFFFF
    return (sign | (new_exp << 10) | ((frac + 0x1000) >> 13)) & 0xFFFF


def _f16_to_f32_bits_py(h):
    """project.rs:160-184, transcribed line by line (returns the f32 bits)."""
    sign = h & 0x8000
    exp = (h >> 10) & 0x1F
    frac = h & 0x3FF
    if exp == 0:
        if frac == 0:
            return sign << 16
        e = 0
        f = frac
        while (f & 0x400) == 0:
            f <<= 1
            e += 1
        f &= 0x3FF
        return (sign << 16) | ((127 - 15 - e) << 23) | (f << 13)
    if exp == 0x1F:
        return (sign << 16) | 0x7F800000 | (frac << 13)
    return (sign << 16) | ((exp + 127 - 15) << 23) | (frac << 13)


def test_layer_offsets_are_o1():
    # state_file.rs:595-605
    descs = sf.build_descriptors([(512, 512), (256, 1024)], [16, 32])
    assert descs[0][3] == sf.HEADER_SIZE + 2 * sf.LAYER_DESC_SIZE
    assert descs[1][3] == descs[0][3] + sf.layer_state_size(512, 512, 16)


def test_galore_half_conversion_matches_transcription(oracle):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32),
        (rng.standard_normal(500) * 1e-5).astype(np.float32),          # f16 subnormal range
        (rng.standard_normal(200) * 7e4).astype(np.float32),           # overflow to inf
        np.array([0.0, -0.0, 1.0, 65504.0, 65520.0, 6.1035156e-05, 5.9604645e-08, np.inf, -np.inf, np.nan],
                 np.float32),
        # mantissa carries with an odd and an even f16 exponent: ORed carry keeps or bumps the exponent
        np.array([np.nextafter(np.float32(2.0), np.float32(0)), np.nextafter(np.float32(4.0), np.float32(0)),
                  np.float32(1.99951171875 + 2 ** -13)], np.float32),
    ])
    got = oracle.galore_f32_to_f16(vals)
    want = np.array([_f32_to_f16_py(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)
    # the carry quirk: just below 2.0 (f16 exponent 15, odd) rounds to 1.0, below 4.0 (exponent 16) to 4.0
    assert oracle.galore_f32_to_f16(np.float32(np.nextafter(np.float32(2.0), np.float32(0))))[0] == 0x3C00
    assert oracle.galore_f32_to_f16(np.float32(np.nextafter(np.float32(4.0), np.float32(0))))[0] == 0x4400
    # f16 -> f32 on every pattern equals the transcription of project.rs:160-184
    # (NaN patterns only by NaN-ness: the ctypes float return quiets signalling NaNs)
    h = np.arange(65536, dtype=np.uint16)
    back = oracle.galore_f16_to_f32(h).view(np.uint32)
    want = np.array([_f16_to_f32_bits_py(int(v)) for v in h], np.uint32)
    nan = (((h >> 10) & 0x1F) == 0x1F) & ((h & 0x3FF) != 0)
    assert np.array_equal(back[~nan], want[~nan])
    assert np.isnan(back[nan].view(np.float32)).all()
    # normal numbers decode exactly; the reference's subnormal branch uses
    # exponent 127 - 15 - e where IEEE needs 127 - 14 - e, so subnormals come
    # back at half their value (kept: it is what the reference reads back)
    ref = h.view(np.float16).astype(np.float32)
    normal = (((h >> 10) & 0x1F) != 0) & (((h >> 10) & 0x1F) != 0x1F)
    assert np.array_equal(back[normal], ref[normal].view(np.uint32))
    sub = (((h >> 10) & 0x1F) == 0) & ((h & 0x3FF) != 0)
    assert np.array_equal(back[sub].view(np.float32), ref[sub] * np.float32(0.5))


def test_header_roundtrip_and_reserved_bytes():
    buf = bytearray(64)
    struct.pack_into("<6IQ", buf, 0, sf.MAGIC, 2, 3, 16, 0, 64, 12345)
    struct.pack_into("<3f", buf, 32, 0.85, 0.99, 1e-6)
    struct.pack_into("<Q", buf, 44, 500)
    h = sf.parse_header(bytes(buf))
    assert (h["magic"], h["version"], h["num_layers"], h["rank"], h["total_size"], h["step_count"]) == \
        (sf.MAGIC, 2, 3, 16, 12345, 500)
    assert math.isclose(h["beta1"], 0.85, rel_tol=1e-6) and h["reserved"] == bytes(12)


def test_state_roundtrip_reference_unit_test(oracle):
    # state_file.rs:626-657: P = 0.01 i, Q = 0.02 i, momentum[0] = 0.5 quantised
    m = n = 64
    r = 4
    p = (0.01 * np.arange(m * r)).astype(np.float32)
    q = (0.02 * np.arange(n * r)).astype(np.float32)
    mom = np.zeros(r * r, np.float32)
    mom[0] = 0.5
    m8, scale_m = oracle.quantize_absmax(mom)
    v8, scale_v = oracle.quantize_absmax(np.zeros(r * r, np.float32))
    descs = sf.build_descriptors([(m, n)], [r])
    buf = bytearray(descs[0][3] + sf.layer_state_size(m, n, r))
    struct.pack_into("<6IQ", buf, 0, sf.MAGIC, 2, 1, r, 0, 64, len(buf))
    struct.pack_into("<3IQ", buf, 64, m, n, r, descs[0][3])
    lay = sf.layer_layout(m, n, r)
    o = descs[0][3]
    buf[o + lay["p"]:o + lay["q"]] = oracle.galore_f32_to_f16(p).tobytes()
    buf[o + lay["q"]:o + lay["m"]] = oracle.galore_f32_to_f16(q).tobytes()
    buf[o + lay["m"]:o + lay["v"]] = m8.tobytes()
    buf[o + lay["v"]:o + lay["scale_m"]] = v8.tobytes()
    struct.pack_into("<ff", buf, o + lay["scale_m"], scale_m, scale_v)
    h, layers = sf.parse(bytes(buf))
    L0 = layers[0]
    assert np.array_equal(L0["m8"], m8) and abs(L0["scale_m"] - scale_m) < 1e-6
    p_read = oracle.galore_f16_to_f32(L0["p_bits"].ravel())
    assert abs(p_read[0] - p[0]) < 1e-3
    assert np.abs(p_read - p).max() <= 2e-3 * np.abs(p).max()
