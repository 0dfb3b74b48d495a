"""ctypes binding of libaeth_galore.so (include/aeth_galore.h).

The shared library is the product; this module only declares its C ABI for
Python callers.  Importing fails loudly when the library is missing -- there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaeth_galore.so")

AETH_OK = 0
AETH_ERR_ARG = -1
AETH_ERR_SHAPE = -2
AETH_ERR_CONFIG = -3
AETH_ERR_UNSUPPORTED = -4
AETH_ERR_NOT_FOUND = -5
AETH_ERR_TIMEOUT = -6
AETH_ERR_LINALG = -7

# bits of the device error word (aeth_device_error_bits)
DEVERR_TIMEOUT_TMA, DEVERR_TIMEOUT_MMA, DEVERR_TIMEOUT_EPI = 1, 2, 4
DEVERR_BAD_ARG, DEVERR_TIMEOUT_PEER = 8, 16
CLIP_HANDLE_BYTES = 64

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
MODE_REF, MODE_B200 = 0, 1
CODEC_PER_TENSOR, CODEC_BLOCK_LINEAR, CODEC_BLOCK_DYNAMIC = 0, 1, 2
WEIGHT_NONE, WEIGHT_F32, WEIGHT_NF4 = 0, 1, 2
REF_GEMM_EXACT, REF_GEMM_SPLIT3 = 0, 1


class GaloreConfig(C.Structure):
    _fields_ = [
        ("mode", C.c_int), ("default_rank", C.c_int), ("attn_rank", C.c_int), ("mlp_rank", C.c_int),
        ("vector_rank", C.c_int), ("switch_interval", C.c_uint64), ("oversampling", C.c_int),
        ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float), ("lr", C.c_float),
        ("weight_decay", C.c_float), ("scale_lr_by_rank", C.c_int), ("max_grad_norm", C.c_float),
        ("state_codec", C.c_int), ("state_block", C.c_int), ("init_projectors", C.c_int),
        ("svd_refresh", C.c_int), ("power_iters", C.c_int), ("grad_dtype", C.c_int),
        ("ref_gemm", C.c_int),
    ]


class ParamSpec(C.Structure):
    _fields_ = [("layer_idx", C.c_uint32), ("name", C.c_char_p), ("m", C.c_int), ("n", C.c_int), ("rank", C.c_int)]


class ParamInfo(C.Structure):
    _fields_ = [("m", C.c_int), ("n", C.c_int), ("rank", C.c_int), ("side", C.c_int),
                ("state_elems", C.c_int64), ("state_blocks", C.c_int64), ("layer_idx", C.c_uint32)]


class WeightRef(C.Structure):
    _fields_ = [("kind", C.c_int), ("data", C.c_void_p), ("absmax", C.c_void_p), ("delta_out", C.c_void_p),
                ("prequant_out", C.c_void_p)]


SQ_HOOK = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p)

_vp, _i, _i64, _f, _u32, _u64, _d = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint32, C.c_uint64, C.c_double

# name -> (restype, argtypes); every function declared in include/aeth_galore.h
SIGNATURES = {
    "galore_project_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "galore_project_backward": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "galore_project_forward_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "galore_quantize_absmax_f32_to_i8": (_i, [_vp, _vp, _vp, _i, _vp]),
    "galore_dequantize_i8_to_f32": (_i, [_vp, _vp, _f, _i, _vp]),
    "doublepass_galore_apply": (None, [_vp, _vp, _vp, _vp, _f, _f, _f, _f, _f, _i, _i]),
    "aeth_galore_config_default": (None, [C.POINTER(GaloreConfig)]),
    "aeth_galore_create": (_i, [C.POINTER(GaloreConfig), C.POINTER(ParamSpec), _i, _i, C.POINTER(_vp)]),
    "aeth_galore_destroy": (_i, [_vp]),
    "aeth_galore_find": (_i, [_vp, _u32, C.c_char_p]),
    "aeth_galore_param_info": (_i, [_vp, _i, C.POINTER(ParamInfo)]),
    "aeth_galore_num_params": (_i, [_vp]),
    "aeth_galore_project_accumulate": (_i, [_vp, _i, _vp, _i, _vp]),
    "aeth_galore_sqnorm_device": (_i, [_vp, _i, _vp, _vp]),
    "aeth_galore_sqnorm": (_i, [_vp, _i, C.POINTER(_d), _vp]),
    "aeth_clip_coeff_device": (_i, [_vp, _i, _f, _vp, _vp, _vp]),
    "aeth_galore_apply_update": (_i, [_vp, _i, _f, _vp, C.POINTER(WeightRef), _vp]),
    "aeth_galore_zero_accum": (_i, [_vp, _i, _vp]),
    "aeth_galore_notify_step": (_i, [_vp, _u64]),
    "aeth_galore_notify_step_async": (_i, [_vp, _u64, _vp]),
    "aeth_galore_version": (_u64, [_vp]),
    "aeth_galore_save_state": (_i, [_vp, C.c_char_p, _vp]),
    "aeth_galore_load_state": (_i, [_vp, C.c_char_p, _vp]),
    "aeth_randomized_svd": (_i, [_vp, _i, _i, _i, _i, _i, _u64, _vp, _vp, _vp]),
    "aeth_randomized_svd_ex": (_i, [_vp, _i, _i, _i, _i, _i, _i, _u64, _i, _vp, _vp, _vp]),
    "aeth_randomized_svd_sketch": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp, _vp]),
    "aeth_rsvd_omega": (_i, [_u64, _i64, _vp, _vp]),
    "aeth_rsvd_jacobi": (_i, [_vp, _i, _vp, _vp]),
    "aeth_galore_step_count": (_u64, [_vp]),
    "aeth_galore_step": (_i, [_vp, _i, C.POINTER(_i), C.POINTER(_vp), _i, C.POINTER(WeightRef), SQ_HOOK, _vp, _vp,
                              _vp]),
    "aeth_galore_project_layer": (_i, [_vp, _i, C.POINTER(_i), C.POINTER(_vp), _i, _vp]),
    "aeth_galore_finish_step": (_i, [_vp, _i, C.POINTER(_i), C.POINTER(WeightRef), SQ_HOOK, _vp, _vp, _vp]),
    "aeth_galore_refresh_layer": (_i, [_vp, _i, C.POINTER(_i), C.POINTER(_vp), _i, _vp]),
    "aeth_galore_projector_buffer": (_i, [_vp, _i, C.POINTER(_vp), C.POINTER(_i), C.POINTER(_i)]),
    "aeth_galore_set_phase_timing": (_i, [_vp, _i]),
    "aeth_galore_phase_times": (_i, [_vp, C.POINTER(_d), C.POINTER(_i)]),
    "aeth_galore_clip_handle": (_i, [_vp, _i, _vp]),
    "aeth_galore_set_clip_group": (_i, [_vp, _i, _i, _vp, _u64]),
    "aeth_galore_set_clip_group_ptrs": (_i, [_vp, _i, _i, C.POINTER(_vp), _u64]),
    "aeth_galore_clip_slots": (_i, [_vp, C.POINTER(_vp)]),
    "aeth_galore_set_projector": (_i, [_vp, _i, _vp, _vp, _vp]),
    "aeth_galore_get_projector": (_i, [_vp, _i, _vp, _vp, _vp]),
    "aeth_galore_get_state": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp]),
    "aeth_galore_set_state": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp]),
    "aeth_galore_get_accum": (_i, [_vp, _i, _vp, _vp]),
    "aeth_nf4_dequant": (_i, [_vp, _vp, _i64, _i, _vp, _i, _vp]),
    "aeth_nf4_quant": (_i, [_vp, _i, _i64, _i, _vp, _vp, _vp]),
    "aeth_int8_quantize": (_i, [_vp, _i64, _i, _i, _i, _vp, _vp, _vp]),
    "aeth_int8_dequantize": (_i, [_vp, _vp, _i64, _i, _i, _i, _vp, _vp]),
    "aeth_dynamic_map": (_i, [_i, C.POINTER(_f)]),
    "aeth_selfcheck": (_i, [_i, C.POINTER(C.c_ulonglong)]),
    "aeth_lomo_sqnorm": (_i, [_vp, _i64, _vp, _vp]),
    "aeth_fc_decode_int8": (_i, [_vp, _i64, _vp, _i64, _i, _vp, _vp]),
    "aeth_fc_decode_nf4": (_i, [_vp, _i64, _f, _vp, _vp]),
    "aeth_bf16_sr_update": (_i, [_vp, _vp, _i64, C.POINTER(C.c_uint64), _vp, _vp]),
    "aeth_lomo_update": (_i, [_vp, _i64, _vp, _f, _f, _f, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "aeth_status_string": (C.c_char_p, [_i]),
    "aeth_last_error": (_i, []),
    "aeth_device_error": (_i, [_i]),
    "aeth_device_error_bits": (_i, [_i, C.POINTER(C.c_uint32)]),
    "aeth_version": (C.c_char_p, []),
}

_lib = None


class AethError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: status {status} ({status_string(status)})")


def load(path: str | None = None):
    """Load the library (once).  Raises ImportError if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(
            f"libaeth_galore.so not found at {p}; build it with `python aethelstream_b200/build.py` "
            "(this package has no CPU fallback)")
    L = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = L
    return L


def status_string(st: int) -> str:
    try:
        return load().aeth_status_string(st).decode()
    except Exception:  # noqa: BLE001 - used while formatting another error
        return "?"


def check(st: int, what: str = "aeth call"):
    if st != AETH_OK:
        raise AethError(st, what)
    return st


def device_error_bits(device: int) -> int:
    """Reads and clears the device error word of `device` (synchronises it):
    the DEVERR_* bits of the bounded waits that gave up."""
    v = C.c_uint32(0)
    check(load().aeth_device_error_bits(device, C.byref(v)), "aeth_device_error_bits")
    return int(v.value)
