"""Streamed-weight decode (flowcast) and the BF16 stochastic-rounding write-back
on the GPU, bit for bit against the oracle's restatements of
flowcast/src/decode.rs and doublepass/src/precision.rs."""
import numpy as np
import pytest
import torch

from tests._gpu import dev, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,num_channels,n_scales", [(100003, 7, 6), (4096, 1, 1), (4099, 0, 0), (37, 5, 5)])
def test_decode_int8_bitexact(oracle, n, num_channels, n_scales):
    from aethelstream_b200 import decode_int8_to_fp16
    rng = np.random.default_rng(n)
    src = rng.integers(-128, 128, n).astype(np.int8)
    scales = (rng.random(max(n_scales, 1)) * 0.05).astype(np.float32)[:n_scales]
    if n_scales > 2:
        scales[1], scales[2] = np.inf, -np.nan  # 0 x inf and NaN products take the host's NaN
    out = decode_int8_to_fp16(dev(src), dev(scales) if n_scales else torch.empty(0, device="cuda"), num_channels)
    ref = oracle.fc_decode_int8(src, scales, num_channels)
    assert np.array_equal(host(out).view(np.uint16), ref)


@pytest.mark.parametrize("absmax", [0.37, 1e10, 1e-9, float("inf"), float("nan"), -float("nan")])
def test_decode_nf4_bitexact(oracle, absmax):
    from aethelstream_b200 import decode_int4_to_fp16
    rng = np.random.default_rng(11)
    src = rng.integers(0, 256, 50001).astype(np.uint8)
    out = decode_int4_to_fp16(dev(src), absmax)
    ref = oracle.fc_decode_int4(src, absmax)
    assert np.array_equal(host(out).view(np.uint16), ref)


def test_bf16_sr_update_bitexact_and_state(oracle):
    from aethelstream_b200 import apply_galore_bf16_update
    rng = np.random.default_rng(5)
    n = 1_000_003
    master = rng.standard_normal(n).astype(np.float32)
    master[:8] = [np.inf, -np.inf, np.nan, 0.0, -0.0, 3.4e38, -3.4e38, 1e-40]
    delta = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    seed = 0xDEAD_BEEF_1234_5678
    tm, td = dev(master), dev(delta)
    bf = torch.empty(n, dtype=torch.int16, device="cuda")
    st = apply_galore_bf16_update(tm, td, seed, bf)
    ref, st_ref = oracle.apply_galore_bf16_update(master, delta, seed)
    got = host(tm)
    assert st == st_ref
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(host(bf).view(np.uint16), (ref.view(np.uint32) >> 16).astype(np.uint16))
    # a second call continues the random stream where the first left it
    st2 = apply_galore_bf16_update(tm, td, st)
    ref2, st2_ref = oracle.apply_galore_bf16_update(ref, delta, st_ref)
    assert st2 == st2_ref and np.array_equal(host(tm).view(np.uint32), ref2.view(np.uint32))


def test_bf16_sr_update_small_and_ragged(oracle):
    from aethelstream_b200 import apply_galore_bf16_update
    rng = np.random.default_rng(6)
    for n in (1, 3, 5, 4097):
        master = rng.standard_normal(n).astype(np.float32)
        delta = (rng.standard_normal(n) * 1e-2).astype(np.float32)
        tm = dev(master)
        st = apply_galore_bf16_update(tm, dev(delta), 0x1111_2222_3333_4444)
        ref, st_ref = oracle.apply_galore_bf16_update(master, delta, 0x1111_2222_3333_4444)
        assert st == st_ref and np.array_equal(host(tm).view(np.uint32), ref.view(np.uint32)), n
