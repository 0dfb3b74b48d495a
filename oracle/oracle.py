"""ctypes/numpy front end for the CPU oracle (``galore_ref.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``.  The product package
(``aethelstream_b200``) never imports it.

Every wrapper names the reference function it restates (paths relative to the
reference project's ``aethelStream/`` directory); the C file carries the
line-level citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_vp = C.c_void_p


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc)."""
    srcs = [os.path.join(_HERE, f) for f in ("galore_ref.c", "doublepass_toy.c", "galore_ref.h")]
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", _HERE, "-B"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "ref_nf4_quantize": (None, [_f32p, C.c_int64, C.c_int, _u8p, _f32p]),
            "ref_nf4_dequant_f32": (None, [_u8p, _f32p, C.c_int64, C.c_int, _f32p]),
            "ref_nf4_dequant_f16": (None, [_u8p, _f32p, C.c_int64, C.c_int, _u16p]),
            "ref_f32_to_f16_rne": (C.c_uint16, [C.c_float]),
            "ref_f32_to_bf16_rne": (C.c_uint16, [C.c_float]),
            "ref_absmax_scale": (C.c_float, [_f32p, C.c_int64]),
            "ref_quantize_absmax": (C.c_float, [_f32p, C.c_int64, _i8p]),
            "ref_dequantize_absmax": (None, [_i8p, C.c_float, C.c_int64, _f32p]),
            "ref_matmul_f32": (None, [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]),
            "ref_project_forward": (None, [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]),
            "ref_project_backward": (None, [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]),
            "ref_projection_roundtrip_error": (C.c_double, [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]),
            "ref_project_forward_rows": (None, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "ref_project_backward_rows": (None, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "ref_adamw_inner_update": (None, [_f32p, _f32p, _f32p, C.c_int64, C.c_float, C.c_float, C.c_float, _f32p]),
            "ref_effective_lr": (C.c_float, [C.c_float, C.c_int, C.c_int]),
            "ref_galore_apply_update": (None, [_f32p, _f32p, _f32p, _i8p, _i8p, _f32p, _f32p, C.c_int, C.c_int,
                                               C.c_int, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float,
                                               C.c_int, _f32p, _f32p]),
            "ref_init_random_projection": (None, [C.c_int, C.c_int, C.c_uint32, _f32p]),
            "ref_rank_for_param": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "ref_clip_coeff": (C.c_float, [C.c_double, C.c_float]),
            "ref_sqnorm_f64": (C.c_double, [_f32p, C.c_int64]),
            "ref_should_switch": (C.c_int, [C.c_uint64, C.c_uint64]),
            "ref_galore_f32_to_f16": (C.c_uint16, [C.c_float]),
            "ref_galore_f16_to_f32": (C.c_float, [C.c_uint16]),
            "ref_rsvd_omega": (None, [C.c_uint64, C.c_int64, _f32p]),
            "ref_rsvd_jacobi": (None, [_f32p, C.c_int, _f32p]),
            "ref_randomized_svd": (C.c_int, [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, _f32p, _f32p]),
            "ref_randomized_svd_sketch": (C.c_int, [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p]),
            "toy_layer_size": (C.c_int64, [C.c_int, C.c_int]),
            "toy_init_layer": (None, [C.c_int, C.c_int, C.c_int, _f32p]),
            "toy_lm_head": (None, [C.c_int, C.c_int, _f32p]),
            "toy_inputs": (None, [C.c_int, C.c_int, C.c_int, _f32p]),
            "toy_labels": (None, [C.c_int, C.c_int, C.c_int, _u32p]),
            "toy_step": (C.c_float, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p,
                                     C.c_int, C.c_int, _u32p, _f32p]),
            "ref_full_adam_apply": (None, [_f32p, _f32p, _f32p, _f32p, C.c_int64, C.c_float, C.c_float, C.c_float,
                                           C.c_float, C.c_float, C.c_int]),
            "b2_dynamic_map": (None, [C.c_int, _f32p]),
            "b2_block_quantize": (None, [_f32p, C.c_int64, C.c_int, C.c_int, C.c_int, _i8p, _f32p]),
            "b2_block_dequantize": (None, [_i8p, _f32p, C.c_int64, C.c_int, C.c_int, C.c_int, _f32p]),
            "b2_side_is_right": (C.c_int, [C.c_int, C.c_int]),
            "b2_project_accumulate": (None, [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]),
            "b2_adam_state": (None, [_f32p, _i8p, _i8p, _f32p, _f32p, C.c_int64, C.c_int, C.c_int, C.c_float,
                                     C.c_float, C.c_float, C.c_float, _vp]),
            "b2_apply_weight": (None, [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _u8p, _f32p, C.c_float, C.c_float,
                                       _u8p, _f32p, _vp, _vp]),
            "b2_nf4_requant": (None, [_f32p, C.c_int64, _u8p, _f32p]),
            "b2_lomo_sqnorm_bf16": (C.c_double, [_u16p, C.c_int64]),
            "b2_lomo_update": (None, [_u16p, C.c_int64, C.c_float, C.c_float, C.c_float, C.c_int, C.c_int, _i8p,
                                      _f32p, _u8p, _f32p, _u8p, _f32p, _vp]),
            "fc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "fc_decode_int8_to_f16": (None, [_i8p, C.c_int64, _f32p, C.c_int64, C.c_int, _u16p]),
            "fc_decode_int4_to_f16": (None, [_u8p, C.c_int64, C.c_float, _u16p]),
            "dp_lcg_next": (C.c_uint16, [C.POINTER(C.c_uint64)]),
            "dp_stochastic_round_to_bf16": (C.c_uint16, [C.c_float, C.c_uint16]),
            "dp_apply_galore_bf16_update": (None, [_f32p, _f32p, C.c_int64, C.POINTER(C.c_uint64)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


NF4_CODES = np.array([
    -1.0, -0.6961928, -0.52507305, -0.3949175, -0.28444138, -0.18477343, -0.09105004, 0.0,
    0.0795803, 0.1609302, 0.2461123, 0.33791524, 0.44070983, 0.562617, 0.72295684, 1.0,
], dtype=np.float32)


# ---- NF4 (shard_engine/python/pipeline/quantizer.py:21-75, shard_engine/src/nf4.rs:37-83) ----
def nf4_quantize(x, block: int = 64):
    x = _c(x, np.float32).ravel()
    n = x.size
    packed = np.zeros((n + 1) // 2, np.uint8)
    absmax = np.zeros((n + block - 1) // block, np.float32)
    lib().ref_nf4_quantize(x, n, block, packed, absmax)
    return packed, absmax


def nf4_dequant_f32(packed, absmax, n: int, block: int = 64):
    out = np.empty(n, np.float32)
    lib().ref_nf4_dequant_f32(_c(packed, np.uint8), _c(absmax, np.float32), n, block, out)
    return out


def nf4_dequant_f16(packed, absmax, n: int, block: int = 64):
    out = np.empty(n, np.uint16)
    lib().ref_nf4_dequant_f16(_c(packed, np.uint8), _c(absmax, np.float32), n, block, out)
    return out.view(np.float16)


def bf16_round(x):
    """Round fp32 values to bf16 (RNE) and return them as fp32."""
    u = _c(x, np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    r = np.where(nan, u | 0x00400000, r).astype(np.uint32)
    return r.view(np.float32).reshape(np.shape(x))


def f32_to_bf16_bits(x):
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- per-tensor absmax INT8 (galore/src/quantize.rs:4-34) ----
def quantize_absmax(x):
    x = _c(x, np.float32).ravel()
    q = np.empty(x.size, np.int8)
    s = lib().ref_quantize_absmax(x, x.size, q)
    return q, np.float32(s)


def dequantize_absmax(q, scale):
    q = _c(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().ref_dequantize_absmax(q, float(scale), q.size, out)
    return out


def absmax_scale(x):
    x = _c(x, np.float32).ravel()
    return np.float32(lib().ref_absmax_scale(x, x.size))


# ---- projections (galore/src/project.rs) ----
def project_forward(g, p, q, m, n, r):
    out = np.zeros(r * r, np.float32)
    lib().ref_project_forward(_c(g, np.float32).ravel(), _c(p, np.float32).ravel(), _c(q, np.float32).ravel(),
                              out, m, n, r)
    return out.reshape(r, r)


def project_backward(nm, p, q, m, n, r):
    out = np.zeros(m * n, np.float32)
    lib().ref_project_backward(_c(nm, np.float32).ravel(), _c(p, np.float32).ravel(), _c(q, np.float32).ravel(),
                               out, m, n, r)
    return out.reshape(m, n)


def projection_roundtrip_error(g, p, q, m, n, r):
    return lib().ref_projection_roundtrip_error(_c(g, np.float32).ravel(), _c(p, np.float32).ravel(),
                                                _c(q, np.float32).ravel(), m, n, r)


def matmul(a, b, m, k, n):
    out = np.zeros(m * n, np.float32)
    lib().ref_matmul_f32(_c(a, np.float32).ravel(), _c(b, np.float32).ravel(), out, m, k, n)
    return out.reshape(m, n)


# ---- Adam (galore/src/adamw.rs) ----
def adamw_inner_update(accum, mom, var, b1=0.9, b2=0.999, eps=1e-8):
    accum = _c(accum, np.float32).ravel()
    mom = _c(mom, np.float32).ravel().copy()
    var = _c(var, np.float32).ravel().copy()
    out = np.empty_like(accum)
    lib().ref_adamw_inner_update(accum, mom, var, accum.size, b1, b2, eps, out)
    return out, mom, var


def galore_apply_update(grad_accum, p, q, m8, v8, scale_m, scale_v, m, n, r, clip,
                        b1=0.9, b2=0.999, eps=1e-8, lr=1e-3, scale_by_rank=False):
    """optimizer.rs:303-362 for one parameter.  Returns (weight_delta, normalized, m8, v8, sm, sv)."""
    m8 = _c(m8, np.int8).ravel().copy()
    v8 = _c(v8, np.int8).ravel().copy()
    sm = np.array([scale_m], np.float32)
    sv = np.array([scale_v], np.float32)
    nrm = np.empty(r * r, np.float32)
    wd = np.empty(m * n, np.float32)
    lib().ref_galore_apply_update(_c(grad_accum, np.float32).ravel(), _c(p, np.float32).ravel(),
                                  _c(q, np.float32).ravel(), m8, v8, sm, sv, m, n, r, clip, b1, b2, eps, lr,
                                  int(scale_by_rank), nrm, wd)
    return wd.reshape(m, n), nrm.reshape(r, r), m8, v8, sm[0], sv[0]


def init_random_projection(rows, cols, seed):
    out = np.empty(rows * cols, np.float32)
    lib().ref_init_random_projection(rows, cols, seed & 0xFFFFFFFF, out)
    return out.reshape(rows, cols)


def rank_for_param(name, m, n, default_rank=16, attn_rank=32, mlp_rank=16, vector_rank=8):
    return lib().ref_rank_for_param(name.encode(), m, n, default_rank, attn_rank, mlp_rank, vector_rank)


def clip_coeff(gsq, max_norm=1.0):
    return np.float32(lib().ref_clip_coeff(float(gsq), max_norm))


def sqnorm_f64(x):
    x = _c(x, np.float32).ravel()
    return lib().ref_sqnorm_f64(x, x.size)


def should_switch(step, interval):
    return bool(lib().ref_should_switch(step, interval))


def rsvd_seed(step):
    """process_pending_svd's seed (optimizer.rs:216-221): step * 0x9E3779B9, wrapping u64."""
    return (int(step) * 0x9E3779B9) & 0xFFFFFFFFFFFFFFFF


def rsvd_omega(seed, count):
    out = np.empty(count, np.float32)
    lib().ref_rsvd_omega(seed, count, out)
    return out


def rsvd_jacobi(a):
    a = _c(a, np.float32).copy()
    n = a.shape[0]
    u = np.empty((n, n), np.float32)
    lib().ref_rsvd_jacobi(a, n, u)
    return u, a


def randomized_svd(g, m, n, r, oversampling, seed, omega=None):
    """(status, P m x r, Q n x r) of randomized_svd_projections; with `omega`
    (n x (r + oversampling) f32) that sketch replaces step 1's draw."""
    g = _c(g, np.float32)
    p = np.zeros((m, r), np.float32)
    q = np.zeros((n, r), np.float32)
    if omega is None:
        st = lib().ref_randomized_svd(g, m, n, r, oversampling, seed, p, q)
    else:
        omega = _c(omega, np.float32)
        assert omega.size == n * (r + oversampling)
        st = lib().ref_randomized_svd_sketch(g, m, n, r, oversampling, omega, p, q)
    return st, p, q


def full_adam_apply(param, grad, m, v, clip, b1, b2, eps, lr, step):
    param = _c(param, np.float32).ravel().copy()
    m = _c(m, np.float32).ravel().copy()
    v = _c(v, np.float32).ravel().copy()
    lib().ref_full_adam_apply(param, _c(grad, np.float32).ravel(), m, v, param.size, clip, b1, b2, eps, lr, step)
    return param, m, v


# ---- B200-mode extensions ----
CODEC_LINEAR, CODEC_DYNAMIC = 0, 1


def dynamic_map(signed: bool):
    out = np.empty(256, np.float32)
    lib().b2_dynamic_map(int(signed), out)
    return out


def block_quantize(x, block=2048, codec=CODEC_LINEAR, signed=True):
    x = _c(x, np.float32).ravel()
    q = np.empty(x.size, np.int8)
    s = np.empty((x.size + block - 1) // block, np.float32)
    lib().b2_block_quantize(x, x.size, block, codec, int(signed), q, s)
    return q, s


def block_dequantize(q, scales, block=2048, codec=CODEC_LINEAR, signed=True):
    q = _c(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().b2_block_dequantize(q, _c(scales, np.float32).ravel(), q.size, block, codec, int(signed), out)
    return out


def side_is_right(m, n):
    return bool(lib().b2_side_is_right(m, n))


def b2_project_accumulate(g, proj, racc, m, n, r):
    racc = _c(racc, np.float32).ravel().copy()
    lib().b2_project_accumulate(_c(g, np.float32).ravel(), _c(proj, np.float32).ravel(), racc, m, n, r)
    return racc


def b2_adam_state(racc, m8, v8, ms, vs, block, codec, clip, b1=0.9, b2=0.999, eps=1e-8):
    racc = _c(racc, np.float32).ravel()
    m8 = _c(m8, np.int8).ravel().copy()
    v8 = _c(v8, np.int8).ravel().copy()
    ms = _c(ms, np.float32).ravel().copy()
    vs = _c(vs, np.float32).ravel().copy()
    nout = np.empty(racc.size, np.float32)
    lib().b2_adam_state(racc, m8, v8, ms, vs, racc.size, block, codec, clip, b1, b2, eps, _ptr(nout))
    return nout, m8, v8, ms, vs


def b2_apply_weight(n_bf16, proj, m, n, r, w_packed, w_absmax, lr, wd=0.0):
    wp = np.empty(m * n // 2, np.uint8)
    wa = np.empty(m * n // 64, np.float32)
    pre = np.empty(m * n, np.float32)
    dw = np.empty(m * n, np.float32)
    lib().b2_apply_weight(_c(n_bf16, np.float32).ravel(), _c(proj, np.float32).ravel(), m, n, r,
                          _c(w_packed, np.uint8).ravel(), _c(w_absmax, np.float32).ravel(), lr, wd, wp, wa,
                          _ptr(pre), _ptr(dw))
    return wp, wa, pre, dw


def nf4_requant(w):
    w = _c(w, np.float32).ravel()
    packed = np.empty((w.size + 1) // 2, np.uint8)
    absmax = np.empty((w.size + 63) // 64, np.float32)
    lib().b2_nf4_requant(w, w.size, packed, absmax)
    return packed, absmax


def lomo_sqnorm(g_bits):
    g = _c(g_bits, np.uint16).ravel()
    return lib().b2_lomo_sqnorm_bf16(g, g.size)


class ReferenceSampler:
    """Times the reference's CPU algorithm for one optimizer step of a set of
    matrices on a bounded row sample (CPU baseline of bench.py).

    Per matrix (galore/src/optimizer.rs:264-362, project.rs:33-58, nf4.rs:37-83):
    Temp = P^T G (only rows i0..i1 of Temp, fraction f of its r rows),
    R = Temp Q for those rows, the r x r Adam update, Temp2 = P N, the weight
    delta rows for fraction f of the m rows, NF4 dequantisation of those weight
    rows and w -= delta.  The O(r m n) loops dominate and scale linearly in f,
    so params/s = f * sum(m n) / time.  Work is split over `threads` Python
    threads (ctypes releases the GIL)."""

    def __init__(self, shapes, r, frac, threads=1, seed=0):
        rng = np.random.default_rng(seed)
        self.r, self.frac, self.threads = r, frac, max(1, threads)
        self.mats = []
        cache = {}
        for (m, n) in shapes:
            if (m, n) not in cache:
                g = (rng.standard_normal((m, n), dtype=np.float32) * np.float32(1e-3))
                p = np.linalg.qr(rng.standard_normal((m, r)))[0].astype(np.float32)
                q = np.linalg.qr(rng.standard_normal((n, r)))[0].astype(np.float32)
                w = (rng.standard_normal(m * n, dtype=np.float32) * np.float32(0.02))
                wp, wa = nf4_quantize(w)
                cache[(m, n)] = (g, p, q, wp, wa)
            self.mats.append((m, n) + cache[(m, n)])
        self.params = sum(m * n for (m, n) in shapes)

    def step(self):
        import concurrent.futures as cf
        lib()
        r, f = self.r, self.frac
        tasks = []
        bufs = []
        for (m, n, g, p, q, wp, wa) in self.mats:
            nfwd = max(1, int(round(r * f)))
            nbwd = max(1, int(round(m * f)))
            temp = np.zeros((r, n), np.float32)
            temp2 = np.zeros((m, r), np.float32)
            out = np.zeros((nbwd, n), np.float32)  # only the sampled rows [0, nbwd) are written
            bufs.append((temp, temp2, out))
            rows = [(i, i + 1) for i in range(nfwd)]
            for (i0, i1) in rows:
                tasks.append(("f", g, p, q, temp, m, n, r, i0, i1))
            chunk = max(1, nbwd // self.threads)
            for i0 in range(0, nbwd, chunk):
                tasks.append(("b", temp2, q, out, m, n, r, i0, min(nbwd, i0 + chunk), wp, wa))

        def run(t):
            if t[0] == "f":
                _, g, p, q, temp, m, n, r_, i0, i1 = t
                lib().ref_project_forward_rows(g.ctypes.data, p.ctypes.data, q.ctypes.data, temp.ctypes.data,
                                               m, n, r_, i0, i1)
            else:
                _, temp2, q, out, m, n, r_, i0, i1, wp, wa = t
                lib().ref_project_backward_rows(temp2.ctypes.data, q.ctypes.data, out.ctypes.data, m, n, r_, i0, i1)
                # weight path for these rows: NF4 dequant (nf4.rs:37-83) and w -= delta
                w = nf4_dequant_f32(wp[i0 * n // 2:i1 * n // 2], wa[i0 * n // 64:i1 * n // 64], (i1 - i0) * n)
                w -= out[i0:i1].ravel()
        with cf.ThreadPoolExecutor(self.threads) as ex:
            list(ex.map(run, tasks))
        # R = Temp Q (sampled rows) and the r x r Adam update (small)
        for (m, n, g, p, q, wp, wa), (temp, temp2, out) in zip(self.mats, bufs):
            nfwd = max(1, int(round(r * f)))
            rr = matmul(temp[:nfwd], q, nfwd, n, r)
            adamw_inner_update(np.resize(rr, r * r), np.zeros(r * r, np.float32), np.zeros(r * r, np.float32))
        return self.params * f


def lomo_update(g_bits, clip, beta, lr, block, codec, mom8, mom_scales, w_packed, w_absmax):
    g = _c(g_bits, np.uint16).ravel()
    n = g.size
    mom8 = _c(mom8, np.int8).ravel().copy()
    ms = _c(mom_scales, np.float32).ravel().copy()
    wp = np.empty((n + 1) // 2, np.uint8)
    wa = np.empty((n + 63) // 64, np.float32)
    pre = np.empty(n, np.float32)
    lib().b2_lomo_update(g, n, clip, beta, lr, block, codec, mom8, ms, _c(w_packed, np.uint8).ravel(),
                         _c(w_absmax, np.float32).ravel(), wp, wa, _ptr(pre))
    return mom8, ms, wp, wa, pre


def galore_f32_to_f16(x):
    """galore's half conversion of the state file (project.rs:137-158), elementwise bits."""
    x = np.asarray(x, np.float32).ravel()
    f = lib().ref_galore_f32_to_f16
    return np.array([f(float(v)) for v in x], np.uint16)


def galore_f16_to_f32(h):
    h = np.asarray(h, np.uint16).ravel()
    f = lib().ref_galore_f16_to_f32
    return np.array([f(int(v)) for v in h], np.float32)


# ---- streamed-weight decode (flowcast/src/decode.rs) and the BF16 write-back (doublepass/src/precision.rs) ----
def fc_f32_to_f16(x: float) -> int:
    return int(lib().fc_f32_to_f16(float(x)))


def fc_decode_int8(src, scales, num_channels: int):
    src = _c(src, np.int8).ravel()
    scales = _c(scales, np.float32).ravel()
    out = np.empty(src.size, np.uint16)
    lib().fc_decode_int8_to_f16(src, src.size, scales, scales.size, num_channels, out)
    return out


def fc_decode_int4(src, absmax: float):
    src = _c(src, np.uint8).ravel()
    out = np.empty(2 * src.size, np.uint16)
    lib().fc_decode_int4_to_f16(src, src.size, float(absmax), out)
    return out


def lcg_next(state: int):
    """(rand16, new_state) of precision.rs:212-217."""
    st = C.c_uint64(state & (2**64 - 1))
    r = lib().dp_lcg_next(C.byref(st))
    return int(r), int(st.value)


def stochastic_round_to_bf16(x: float, rand_bits: int) -> int:
    return int(lib().dp_stochastic_round_to_bf16(float(x), int(rand_bits)))


def apply_galore_bf16_update(master, delta, state: int):
    """(new master, new rng state) of apply_galore_bf16_update (precision.rs:184-202)."""
    m = _c(master, np.float32).ravel().copy()
    d = _c(delta, np.float32).ravel()
    st = C.c_uint64(state & (2**64 - 1))
    lib().dp_apply_galore_bf16_update(m, d, m.size, C.byref(st))
    return m, int(st.value)


# ---- the galore tests' toy transformer (doublepass_toy.c) ----
class ToyModel:
    """The model galore/tests/common/mod.rs trains (doublepass Model::new with
    BlockWeights::from_formula_layered), its inputs, labels and LM head, and one
    step's loss and gradients in the reference's f32 arithmetic."""

    NAMES = ("d_rms1_w", "d_wq", "d_wk", "d_wv", "d_wo", "d_rms2_w", "d_wg", "d_wu", "d_wd")

    def __init__(self, d, n_heads, d_ff, seq_len=4, batch=1, n_layers=2, vocab=64, chunk_size=256):
        self.d, self.h, self.ff, self.s, self.b, self.nl, self.vocab, self.chunk = (d, n_heads, d_ff, seq_len, batch,
                                                                                 n_layers, vocab, chunk_size)
        self.lf = int(lib().toy_layer_size(d, d_ff))
        self.w = np.empty(self.nl * self.lf, np.float32)
        for li in range(self.nl):
            blk = np.empty(self.lf, np.float32)
            lib().toy_init_layer(d, d_ff, li, blk)
            self.w[li * self.lf:(li + 1) * self.lf] = blk
        self.lm = np.empty(vocab * d, np.float32)
        lib().toy_lm_head(vocab, d, self.lm)
        self.x = np.empty(seq_len * batch * d, np.float32)
        lib().toy_inputs(d, seq_len, batch, self.x)
        self.labels = np.empty(seq_len * batch, np.uint32)
        lib().toy_labels(seq_len, batch, vocab, self.labels)
        d_, ff = d, d_ff
        self.shapes = [(1, d_), (d_, d_), (d_, d_), (d_, d_), (d_, d_), (1, d_), (ff, d_), (ff, d_), (d_, ff)]

    def param_specs(self):
        """(layer, name, m, n) in the order of galore/tests/common/mod.rs:73-89."""
        return [(li, nm, m, n) for li in range(self.nl) for nm, (m, n) in zip(self.NAMES, self.shapes)]

    def _slot(self, li, name):
        off = li * self.lf
        for nm, (m, n) in zip(self.NAMES, self.shapes):
            if nm == name:
                return off, m * n
            off += m * n
        raise KeyError(name)

    def step(self):
        """(loss, {(layer, name): gradient m x n})."""
        g = np.empty_like(self.w)
        loss = lib().toy_step(self.d, self.h, self.ff, self.s, self.b, self.nl, self.w, self.x, self.lm, self.vocab,
                              self.chunk, self.labels, g)
        out = {}
        for li, nm, m, n in self.param_specs():
            off, cnt = self._slot(li, nm)
            out[(li, nm)] = g[off:off + cnt].reshape(m, n)
        return float(np.float32(loss)), out

    def apply_delta(self, li, name, delta):
        """apply_weight_delta (common/mod.rs:106-111): w -= delta, f32."""
        off, cnt = self._slot(li, name)
        self.w[off:off + cnt] -= np.asarray(delta, np.float32).ravel()
