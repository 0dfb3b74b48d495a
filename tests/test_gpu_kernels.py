"""GPU parity of the stand-alone kernels against the CPU oracle, through the
C ABI: NF4 dequant/quant (bit-exact), INT8 codecs (bit-exact), the
reference-compatible quantise/apply symbols, and LOMO."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from tests._gpu import DEV, bf16_dev_from_bits, dev, host, ptr, rel_fro, stream

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "nf4_golden.npz")


@pytest.fixture(scope="module")
def L():
    from aethelstream_b200 import _lib
    return _lib


@pytest.fixture(scope="module")
def lib(L):
    return L.load()


def _nf4_inputs(oracle):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(1 << 20) * 0.02).astype(np.float32)
    return x, *oracle.nf4_quantize(x)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_nf4_dequant_bitexact(oracle, L, lib, dtype):
    x, packed, absmax = _nf4_inputs(oracle)
    n = x.size
    ref = oracle.nf4_dequant_f32(packed, absmax, n)
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dtype]
    code = {"f32": L.DTYPE_F32, "f16": L.DTYPE_F16, "bf16": L.DTYPE_BF16}[dtype]
    out = torch.empty(n, dtype=tdt, device=DEV)
    p, a = dev(packed), dev(absmax)
    assert lib.aeth_nf4_dequant(ptr(p), ptr(a), n, 64, ptr(out), code, stream()) == 0
    got = out.float().cpu().numpy()
    expect = torch.from_numpy(ref).to(tdt).float().numpy()  # RNE cast of the exact product
    assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))


def test_nf4_dequant_generic_path(oracle, L, lib):
    """Odd length and block size 32 take the generic kernel (nf4.rs:37-83 partial block)."""
    rng = np.random.default_rng(12)
    n = 1001
    x = rng.standard_normal(n).astype(np.float32)
    packed, absmax = oracle.nf4_quantize(x, block=32)
    ref = oracle.nf4_dequant_f16(packed, absmax, n, block=32)
    out = torch.empty(n, dtype=torch.float16, device=DEV)
    assert lib.aeth_nf4_dequant(ptr(dev(packed)), ptr(dev(absmax)), n, 32, ptr(out), L.DTYPE_F16, stream()) == 0
    assert np.array_equal(host(out).view(np.uint16), ref.view(np.uint16))


def test_nf4_quant_reference_golden(L, lib):
    """Every fixture made by the reference quantiser, through the GPU."""
    z = np.load(GOLDEN)
    for name in sorted({k.split("__")[0] for k in z.files}):
        x = z[f"{name}__input"]
        n = x.size
        packed = torch.zeros((n + 1) // 2, dtype=torch.uint8, device=DEV)
        absmax = torch.zeros((n + 63) // 64, dtype=torch.float32, device=DEV)
        assert lib.aeth_nf4_quant(ptr(dev(x)), L.DTYPE_F32, n, 64, ptr(packed), ptr(absmax), stream()) == 0
        assert np.array_equal(host(packed), z[f"{name}__packed"]), name
        assert np.array_equal(host(absmax).view(np.uint32), z[f"{name}__absmax"].view(np.uint32)), name


def test_nf4_quant_nonfinite_generic_block(oracle, L, lib):
    """NaN / inf through the generic path (block 32, odd length) as the
    reference quantiser treats them (absmax NaN propagates; codes from argmin)."""
    rng = np.random.default_rng(77)
    x = (rng.standard_normal(333) * 0.02).astype(np.float32)
    x[[1, 40, 41, 100, 200]] = [np.nan, np.inf, -np.inf, np.inf, np.nan]
    n = x.size
    packed = torch.zeros((n + 1) // 2, dtype=torch.uint8, device=DEV)
    absmax = torch.zeros((n + 31) // 32, dtype=torch.float32, device=DEV)
    assert lib.aeth_nf4_quant(ptr(dev(x)), L.DTYPE_F32, n, 32, ptr(packed), ptr(absmax), stream()) == 0
    p_ref, a_ref = oracle.nf4_quantize(x, block=32)
    assert np.array_equal(host(packed), p_ref)
    assert np.array_equal(host(absmax).view(np.uint32), a_ref.view(np.uint32))


def _boundary_heavy(oracle, nblocks, seed):
    """Blocks whose values sit on, or one ulp either side of, the decision
    midpoints (scaled by the block absmax) -- the cases the fast classifier
    must hand to the exact path."""
    rng = np.random.default_rng(seed)
    codes = oracle.NF4_CODES
    mids = ((codes[:-1] + codes[1:]) * np.float32(0.5)).astype(np.float32)
    out = np.empty((nblocks, 64), np.float32)
    for b in range(nblocks):
        a = np.float32(rng.uniform(1e-3, 10.0))
        v = mids[rng.integers(0, 15, 64)] * a
        v = np.where(rng.random(64) < 0.3, np.nextafter(v, np.float32(np.inf)), v)
        v = np.where(rng.random(64) < 0.3, np.nextafter(v, np.float32(-np.inf)), v).astype(np.float32)
        v[rng.integers(0, 64)] = a if rng.random() < 0.5 else -a
        out[b] = v
    return out.ravel()


@pytest.mark.parametrize("kind", ["gauss", "boundary", "bf16", "f16"])
def test_nf4_quant_bitexact(oracle, L, lib, kind):
    rng = np.random.default_rng(13)
    if kind == "boundary":
        x = _boundary_heavy(oracle, 4096, 14)
    else:
        x = (rng.standard_normal(1 << 20) * 0.02).astype(np.float32)
    tdt, code = torch.float32, L.DTYPE_F32
    if kind == "bf16":
        tdt, code = torch.bfloat16, L.DTYPE_BF16
    elif kind == "f16":
        tdt, code = torch.float16, L.DTYPE_F16
    xt = dev(x).to(tdt)
    xr = xt.float().cpu().numpy()  # the values the kernel sees
    n = x.size
    packed = torch.empty(n // 2, dtype=torch.uint8, device=DEV)
    absmax = torch.empty(n // 64, dtype=torch.float32, device=DEV)
    assert lib.aeth_nf4_quant(ptr(xt), code, n, 64, ptr(packed), ptr(absmax), stream()) == 0
    p_ref, a_ref = oracle.nf4_quantize(xr)
    assert np.array_equal(host(absmax).view(np.uint32), a_ref.view(np.uint32))
    assert np.array_equal(host(packed), p_ref)


@pytest.mark.parametrize("codec,signed", [(0, True), (1, True), (1, False), (2, True), (2, False)])
def test_int8_codecs_bitexact(oracle, L, lib, codec, signed):
    rng = np.random.default_rng(15)
    n = 3 * 2048 + 512
    x = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    if not signed:
        x = np.abs(x)
    nb = 1 if codec == L.CODEC_PER_TENSOR else (n + 2047) // 2048
    q = torch.empty(n, dtype=torch.int8, device=DEV)
    s = torch.empty(nb, dtype=torch.float32, device=DEV)
    assert lib.aeth_int8_quantize(ptr(dev(x)), n, codec, 2048, int(signed), ptr(q), ptr(s), stream()) == 0
    if codec == L.CODEC_PER_TENSOR:
        q_ref, s_ref = oracle.quantize_absmax(x)
        s_ref = np.array([s_ref], np.float32)
        rec_ref = oracle.dequantize_absmax(q_ref, s_ref[0])
    else:
        oc = oracle.CODEC_LINEAR if codec == L.CODEC_BLOCK_LINEAR else oracle.CODEC_DYNAMIC
        q_ref, s_ref = oracle.block_quantize(x, 2048, oc, signed)
        rec_ref = oracle.block_dequantize(q_ref, s_ref, 2048, oc, signed)
    assert np.array_equal(host(q), q_ref)
    assert np.array_equal(host(s).view(np.uint32), s_ref.view(np.uint32))
    out = torch.empty(n, dtype=torch.float32, device=DEV)
    assert lib.aeth_int8_dequantize(ptr(q), ptr(s), n, codec, 2048, int(signed), ptr(out), stream()) == 0
    assert np.array_equal(host(out).view(np.uint32), rec_ref.view(np.uint32))


def test_reference_quantize_symbols(oracle, lib):
    """galore_quantize_absmax_f32_to_i8 / galore_dequantize_i8_to_f32
    (quantize_state.cuh:12-26) with the live CPU path's rounding."""
    rng = np.random.default_rng(16)
    n = 100_003
    x = (rng.standard_normal(n) * 3e-4).astype(np.float32)
    x[17] = np.float32(0.0)
    q = torch.empty(n, dtype=torch.int8, device=DEV)
    scale = torch.empty(1, dtype=torch.float32, device=DEV)
    assert lib.galore_quantize_absmax_f32_to_i8(ptr(dev(x)), ptr(q), ptr(scale), n, stream()) == 0
    q_ref, s_ref = oracle.quantize_absmax(x)
    assert np.array_equal(host(q), q_ref) and host(scale)[0] == s_ref
    out = torch.empty(n, dtype=torch.float32, device=DEV)
    assert lib.galore_dequantize_i8_to_f32(ptr(q), ptr(out), float(s_ref), n, stream()) == 0
    assert np.array_equal(host(out), oracle.dequantize_absmax(q_ref, s_ref))
    # zero tensor: scale 1.0 (quantize.rs:8-9)
    z = torch.zeros(64, device=DEV)
    assert lib.galore_quantize_absmax_f32_to_i8(ptr(z), ptr(q), ptr(scale), 64, stream()) == 0
    assert host(scale)[0] == 1.0


@pytest.mark.parametrize("step", [0, 5])
def test_doublepass_galore_apply(oracle, lib, step):
    rng = np.random.default_rng(17)
    n = 50_000
    param = rng.standard_normal(n).astype(np.float32)
    grad = (rng.standard_normal(n) * 1e-2).astype(np.float32)
    m = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * 1e-5).astype(np.float32)
    tp, tg, tm, tv = dev(param), dev(grad), dev(m), dev(v)
    torch.cuda.synchronize()
    lib.doublepass_galore_apply(ptr(tp), ptr(tg), ptr(tm), ptr(tv), 0.75, 0.9, 0.999, 1e-8, 1e-3, n, step)
    assert lib.aeth_last_error() == 0
    torch.cuda.synchronize()
    p_ref, m_ref, v_ref = oracle.full_adam_apply(param, grad, m, v, 0.75, 0.9, 0.999, 1e-8, 1e-3, step)
    assert np.array_equal(host(tm), m_ref) and np.array_equal(host(tv), v_ref)
    assert np.array_equal(host(tp), p_ref)


@pytest.mark.parametrize("codec", [1, 2])
def test_lomo_step(oracle, L, lib, codec):
    rng = np.random.default_rng(18)
    n = 1 << 18
    g_bits = oracle.f32_to_bf16_bits((rng.standard_normal(n) * 1e-3).astype(np.float32))
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    wp, wa = oracle.nf4_quantize(w)
    mom = (rng.standard_normal(n) * 1e-4).astype(np.float32)
    oc = oracle.CODEC_LINEAR if codec == L.CODEC_BLOCK_LINEAR else oracle.CODEC_DYNAMIC
    mom8, ms = oracle.block_quantize(mom, 2048, oc, True)
    tg = bf16_dev_from_bits(g_bits)
    twp, twa, tm8, tms = dev(wp), dev(wa), dev(mom8), dev(ms)
    sq = torch.zeros(1, dtype=torch.float64, device=DEV)
    pre = torch.empty(n, dtype=torch.float32, device=DEV)
    assert lib.aeth_lomo_sqnorm(ptr(tg), n, ptr(sq), stream()) == 0
    assert lib.aeth_lomo_update(ptr(tg), n, ptr(sq), 1.0, 1e-3, 0.9, codec, 2048, ptr(tm8), ptr(tms), ptr(twp),
                                ptr(twa), ptr(pre), stream()) == 0
    sq_gpu = float(host(sq)[0])
    sq_ref = oracle.lomo_sqnorm(g_bits)
    assert abs(sq_gpu - sq_ref) <= 1e-12 * sq_ref
    clip = oracle.clip_coeff(sq_gpu, 1.0)  # same clip the kernel derived from the same sum
    m8_ref, ms_ref, wp_ref, wa_ref, pre_ref = oracle.lomo_update(g_bits, float(clip), 0.9, 1e-3, 2048, oc, mom8, ms,
                                                                 wp, wa)
    assert np.array_equal(host(pre), pre_ref)
    assert np.array_equal(host(tm8), m8_ref) and np.array_equal(host(tms), ms_ref)
    assert np.array_equal(host(twp), wp_ref) and np.array_equal(host(twa), wa_ref)
    assert rel_fro(host(pre), w) < 0.2


@pytest.mark.parametrize("which", [0, 1, 2, 3], ids=["dmap_signed", "dmap_unsigned", "adam_dir", "nf4_classify"])
def test_fast_paths_exhaustive(lib, which):
    """Over all 2^32 float bit patterns: the bucket-table dynamic-map encoder
    of the Adam and LOMO kernels returns the binary search's code, and the
    approximate Adam direction rounds to the same bf16 as IEEE sqrt/div.  Over
    every |x| <= absmax for six block scales: the fused epilogues' NF4
    classifier returns quantizer.py's argmin code."""
    bad = C.c_ulonglong(12345)
    assert lib.aeth_selfcheck(which, C.byref(bad)) == 0
    assert bad.value == 0
    assert lib.aeth_selfcheck(4, C.byref(bad)) == -1  # unknown check


def test_lomo_python_wrappers(oracle, L):
    """lomo_sqnorm / lomo_update (the Python face of aeth_lomo_*) against the oracle's LOMO step."""
    from aethelstream_b200 import LomoState, lomo_sqnorm, lomo_update, nf4_quantize
    rng = np.random.default_rng(19)
    n = 1 << 16
    g_bits = oracle.f32_to_bf16_bits((rng.standard_normal(n) * 1e-3).astype(np.float32))
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    W = nf4_quantize(dev(w))
    wp, wa = host(W.packed), host(W.absmax)
    st = LomoState(n, DEV)
    g = bf16_dev_from_bits(g_bits)
    sq = lomo_sqnorm(g, st)
    lomo_update(g, W, st, max_norm=1.0, lr=1e-3, beta=0.9)
    clip = oracle.clip_coeff(float(host(sq)[0]), 1.0)
    m8, ms, wp_ref, wa_ref, _ = oracle.lomo_update(g_bits, float(clip), 0.9, 1e-3, 2048, oracle.CODEC_DYNAMIC,
                                                   np.zeros(n, np.int8), np.zeros(n // 2048, np.float32), wp, wa)
    assert np.array_equal(host(st.mom8), m8) and np.array_equal(host(st.scales), ms)
    assert np.array_equal(host(W.packed), wp_ref) and np.array_equal(host(W.absmax), wa_ref)
