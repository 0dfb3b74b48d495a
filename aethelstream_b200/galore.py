"""Host-side mirror of the reference `galore` crate's operator surface.

``GaLoreOptimizer`` implements the methods of ``doublepass::OptimizerBackend``
(doublepass/src/lib.rs:62-107) as ``galore::GaLoreOptimizer`` does
(galore/src/optimizer.rs:81-403), with the same names, argument meaning and
error behaviour (unknown keys and wrong-sized gradients are ignored, as the
reference does), on top of libaeth_galore's C ABI.  Device memory and streams
come from torch; all arithmetic runs in the library's CUDA kernels.

``deferred_apply_with_clip`` mirrors doublepass/src/hook.rs:115-259.
Reference paths are relative to the reference project's aethelStream/.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass, field

import torch

from . import _lib as L


class ProjectorKind(enum.Enum):
    """doublepass/src/hook.rs:44-68"""
    ORTHONORMAL = 0
    RANDOM = 1
    NONE = 2


@dataclass
class AdamWConfig:
    """galore/src/adamw.rs:8-34"""
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    lr: float = 1e-3
    weight_decay: float = 0.0
    scale_lr_by_rank: bool = False


@dataclass
class LayerRankConfig:
    """galore/src/layer_rank.rs:8-40"""
    default_rank: int = 16
    attn_rank: int = 32
    mlp_rank: int = 16
    vector_rank: int = 8

    def rank_for_param(self, param_name: str, m: int, n: int) -> int:
        if param_name in ("d_wq", "d_wk", "d_wv", "d_wo"):
            base = self.attn_rank
        elif param_name in ("d_wg", "d_wu", "d_wd"):
            base = self.mlp_rank
        elif param_name in ("d_rms1_w", "d_rms2_w"):
            base = self.vector_rank
        else:
            base = self.default_rank
        return max(min(base, max(m, 1), max(n, 1)), 1)


@dataclass
class GaLoreConfig:
    """galore/src/optimizer.rs:35-61 plus the B200-mode options.

    mode "ref": two-sided projection, fp32, per-tensor INT8 (the reference).
    mode "b200": one-sided projection on the smaller dimension, bf16 tensor
    cores, blockwise INT8 state ("linear" or "dynamic"), fused NF4 weight write.
    """
    rank: int = 16
    layer_ranks: LayerRankConfig = field(default_factory=LayerRankConfig)
    switch_interval: int = 200
    oversampling: int = 10
    adam: AdamWConfig = field(default_factory=AdamWConfig)
    mode: str = "ref"
    state_codec: str = "per_tensor"
    state_block: int = 2048
    max_grad_norm: float = 1.0
    init_projectors: bool = True
    # subspace refresh in notify_step as the reference (False: fixed projectors)
    svd_refresh: bool = True
    power_iters: int = 0
    # B200: dtype of the gradients ("bf16", "f32", "f16"); f32 / f16 set up the
    # exact split path's buffers at construction, so no step allocates
    grad_dtype: str = "bf16"
    # REF: "exact" (the reference's loop order, bit for bit, CUDA cores) or
    # "split3" (tensor cores on exact bf16 terms, fp32 accuracy)
    ref_gemm: str = "exact"

    def to_c(self) -> L.GaloreConfig:
        c = L.GaloreConfig()
        L.load().aeth_galore_config_default(C.byref(c))
        c.mode = {"ref": L.MODE_REF, "b200": L.MODE_B200}[self.mode]
        c.default_rank = self.layer_ranks.default_rank
        c.attn_rank = self.layer_ranks.attn_rank
        c.mlp_rank = self.layer_ranks.mlp_rank
        c.vector_rank = self.layer_ranks.vector_rank
        c.switch_interval = self.switch_interval
        c.oversampling = self.oversampling
        c.beta1, c.beta2, c.eps, c.lr = self.adam.beta1, self.adam.beta2, self.adam.eps, self.adam.lr
        c.weight_decay = self.adam.weight_decay
        c.scale_lr_by_rank = int(self.adam.scale_lr_by_rank)
        c.max_grad_norm = self.max_grad_norm
        # REF mode is per-tensor INT8 (quantize.rs); B200 mode is blockwise.
        codec = "per_tensor" if self.mode == "ref" else ("dynamic" if self.state_codec == "dynamic" else "linear")
        c.state_codec = {"per_tensor": L.CODEC_PER_TENSOR, "linear": L.CODEC_BLOCK_LINEAR,
                         "dynamic": L.CODEC_BLOCK_DYNAMIC}[codec]
        c.state_block = self.state_block
        c.init_projectors = int(self.init_projectors)
        c.svd_refresh = int(self.svd_refresh)
        c.power_iters = self.power_iters
        c.grad_dtype = {"f32": L.DTYPE_F32, "f16": L.DTYPE_F16, "bf16": L.DTYPE_BF16}[self.grad_dtype]
        c.ref_gemm = {"exact": L.REF_GEMM_EXACT, "split3": L.REF_GEMM_SPLIT3}[self.ref_gemm]
        return c


_DTYPES = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16, torch.bfloat16: L.DTYPE_BF16}


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


@dataclass
class NF4Tensor:
    """NF4 weight: 64-element blocks, fp32 absmax, high nibble = even element
    (shard_engine/src/nf4.rs:25-83)."""
    packed: torch.Tensor   # uint8, numel/2
    absmax: torch.Tensor   # float32, numel/64
    shape: tuple

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def nf4_quantize(x: torch.Tensor, block: int = 64) -> NF4Tensor:
    """quantize_nf4 (shard_engine/python/pipeline/quantizer.py:21-53) on the GPU, bit-exact."""
    x = x.contiguous()
    n = x.numel()
    packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=x.device)
    absmax = torch.empty((n + block - 1) // block, dtype=torch.float32, device=x.device)
    L.check(L.load().aeth_nf4_quant(_ptr(x), _DTYPES[x.dtype], n, block, _ptr(packed), _ptr(absmax),
                                    C.c_void_p(_stream_handle())), "aeth_nf4_quant")
    return NF4Tensor(packed, absmax, tuple(x.shape))


def nf4_dequantize(t: NF4Tensor, dtype: torch.dtype = torch.float16, block: int = 64) -> torch.Tensor:
    """dequant_nf4_into (shard_engine/src/nf4.rs:37-83) / dequantize_nf4 (quantizer.py:55-75)."""
    out = torch.empty(t.shape, dtype=dtype, device=t.packed.device)
    L.check(L.load().aeth_nf4_dequant(_ptr(t.packed), _ptr(t.absmax), t.numel, block, _ptr(out), _DTYPES[dtype],
                                      C.c_void_p(_stream_handle())), "aeth_nf4_dequant")
    return out


def randomized_svd(g: torch.Tensor, rank: int, oversampling: int = 10, seed: int = 42, power_iters: int = 0,
                   want_p: bool = True, want_q: bool = True):
    """randomized_svd_projections (galore/src/randomized_svd.rs:76-149) on the
    device: (P m x r, Q n x r) f32 for the f32 matrix g (m x n).  Raises
    AethError(AETH_ERR_CONFIG) for rank 0 or rank + oversampling > min(m, n)
    and AethError(AETH_ERR_LINALG) for a rank-deficient sketch."""
    g = g.contiguous()
    if g.dtype != torch.float32 or g.dim() != 2:
        raise ValueError("g must be a 2-D float32 device tensor")
    m, n = g.shape
    p = torch.empty(m, rank, dtype=torch.float32, device=g.device) if want_p else None
    q = torch.empty(n, rank, dtype=torch.float32, device=g.device) if want_q else None
    L.check(L.load().aeth_randomized_svd(_ptr(g), m, n, rank, oversampling, power_iters, seed & (2**64 - 1),
                                         _ptr(p), _ptr(q), C.c_void_p(_stream_handle())), "aeth_randomized_svd")
    return p, q


def randomized_svd_fast(g: torch.Tensor, rank: int, oversampling: int = 10, seed: int = 42, power_iters: int = 0,
                        want_p: bool = True, want_q: bool = True):
    """randomized_svd with every product on the tensor cores over exact bf16
    terms (fp32-accurate, not the reference's summation order); g is a float32
    or bfloat16 device matrix."""
    g = g.contiguous()
    if g.dtype not in (torch.float32, torch.bfloat16) or g.dim() != 2:
        raise ValueError("g must be a 2-D float32 or bfloat16 device tensor")
    m, n = g.shape
    p = torch.empty(m, rank, dtype=torch.float32, device=g.device) if want_p else None
    q = torch.empty(n, rank, dtype=torch.float32, device=g.device) if want_q else None
    L.check(L.load().aeth_randomized_svd_ex(_ptr(g), _DTYPES[g.dtype], m, n, rank, oversampling, power_iters,
                                            seed & (2**64 - 1), 1, _ptr(p), _ptr(q), C.c_void_p(_stream_handle())),
            "aeth_randomized_svd_ex")
    return p, q


def randomized_svd_sketch(g: torch.Tensor, rank: int, oversampling: int, omega: torch.Tensor, fast: bool = False,
                          want_p: bool = True, want_q: bool = True):
    """randomized_svd_projections (galore/src/randomized_svd.rs:95-149) from
    the caller's sketch omega (n x (rank + oversampling) float32 on the
    device) instead of the seeded draw.  With fast=False the products and the
    Gram-Schmidt run in the reference's own order, so the sketch the
    reference drew gives its P and Q bit for bit."""
    g = g.contiguous()
    omega = omega.contiguous()
    if g.dtype not in (torch.float32, torch.bfloat16) or g.dim() != 2:
        raise ValueError("g must be a 2-D float32 or bfloat16 device tensor")
    m, n = g.shape
    if omega.dtype != torch.float32 or omega.shape != (n, rank + oversampling) or omega.device != g.device:
        raise ValueError("omega must be a float32 (n, rank + oversampling) tensor on g's device")
    p = torch.empty(m, rank, dtype=torch.float32, device=g.device) if want_p else None
    q = torch.empty(n, rank, dtype=torch.float32, device=g.device) if want_q else None
    L.check(L.load().aeth_randomized_svd_sketch(_ptr(g), _DTYPES[g.dtype], m, n, rank, oversampling, _ptr(omega),
                                                int(bool(fast)), _ptr(p), _ptr(q), C.c_void_p(_stream_handle())),
            "aeth_randomized_svd_sketch")
    return p, q


def decode_int8_to_fp16(src: torch.Tensor, scales: torch.Tensor, num_channels: int) -> torch.Tensor:
    """QuantizedDecoder::decode_int8_to_fp16 (flowcast/src/decode.rs:63-86) on
    the device: int8 src, per-channel f32 scales -> float16 (flowcast's
    truncating conversion)."""
    src = src.contiguous()
    out = torch.empty(src.numel(), dtype=torch.float16, device=src.device)
    sc = scales.contiguous().float()
    L.check(L.load().aeth_fc_decode_int8(_ptr(src), src.numel(), _ptr(sc), sc.numel(), num_channels, _ptr(out),
                                         C.c_void_p(_stream_handle())), "aeth_fc_decode_int8")
    return out


def decode_int4_to_fp16(src: torch.Tensor, absmax: float) -> torch.Tensor:
    """QuantizedDecoder::decode_int4_to_fp16 (decode.rs:88-104): packed NF4
    bytes, low nibble first, one absmax -> float16 (2 values per byte)."""
    src = src.contiguous()
    out = torch.empty(2 * src.numel(), dtype=torch.float16, device=src.device)
    L.check(L.load().aeth_fc_decode_nf4(_ptr(src), src.numel(), float(absmax), _ptr(out),
                                        C.c_void_p(_stream_handle())), "aeth_fc_decode_nf4")
    return out


def apply_galore_bf16_update(master: torch.Tensor, delta: torch.Tensor, rng_state: int,
                             bf16_out: torch.Tensor | None = None) -> int:
    """apply_galore_bf16_update (doublepass/src/precision.rs:184-202) on the
    device, in place on the f32 master weights; returns the advanced LCG state."""
    st = C.c_uint64(rng_state & (2**64 - 1))
    L.check(L.load().aeth_bf16_sr_update(_ptr(master), _ptr(delta), master.numel(), C.byref(st), _ptr(bf16_out),
                                         C.c_void_p(_stream_handle())), "aeth_bf16_sr_update")
    return int(st.value)


class LomoState:
    """INT8 blockwise momentum of a LOMO-updated NF4 tensor (codec 1: linear,
    2: dynamic map; one fp32 scale per `block` elements)."""

    def __init__(self, n: int, device, codec: int = L.CODEC_BLOCK_DYNAMIC, block: int = 2048):
        self.n, self.codec, self.block = n, codec, block
        self.mom8 = torch.zeros(n, dtype=torch.int8, device=device)
        fill = 1.0 if codec == L.CODEC_BLOCK_LINEAR else 0.0
        self.scales = torch.full(((n + block - 1) // block,), fill, dtype=torch.float32, device=device)
        self.sq = torch.zeros(1, dtype=torch.float64, device=device)


def lomo_sqnorm(grad: torch.Tensor, state: LomoState, accumulate: bool = False) -> torch.Tensor:
    """Pass 1 of the LOMO step: state.sq (+)= sum(g^2) in f64 over the bf16
    gradient.  Returns state.sq, which a multi-GPU caller all-reduces before
    lomo_update."""
    if not accumulate:
        state.sq.zero_()
    L.check(L.load().aeth_lomo_sqnorm(_ptr(grad), grad.numel(), _ptr(state.sq), C.c_void_p(_stream_handle())),
            "aeth_lomo_sqnorm")
    return state.sq


def lomo_update(grad: torch.Tensor, weight: NF4Tensor, state: LomoState, max_norm: float, lr: float,
                beta: float = 0.9, prequant_out: torch.Tensor | None = None) -> None:
    """Pass 2: clip from state.sq, INT8 momentum m = beta m + clip g, w -= lr m,
    NF4 requantisation of w in place (aeth_lomo_update)."""
    L.check(L.load().aeth_lomo_update(_ptr(grad), grad.numel(), _ptr(state.sq), float(max_norm), float(lr), float(beta),
                                      state.codec, state.block, _ptr(state.mom8), _ptr(state.scales),
                                      _ptr(weight.packed), _ptr(weight.absmax), _ptr(prequant_out),
                                      C.c_void_p(_stream_handle())), "aeth_lomo_update")


class GaLoreOptimizer:
    """galore::GaLoreOptimizer on the B200 library (one device per instance)."""

    def __init__(self, config: GaLoreConfig, param_specs, device: int | None = None):
        self.config = config
        self.device = torch.cuda.current_device() if device is None else device
        self._lib = L.load()
        specs = (L.ParamSpec * max(len(param_specs), 1))()
        self._names = []
        for i, spec in enumerate(param_specs):
            li, name, m, n = spec[:4]
            rank = spec[4] if len(spec) > 4 else 0
            bname = name.encode()
            self._names.append(bname)  # keep alive for the call
            specs[i] = L.ParamSpec(li, bname, m, n, rank)
        self._cfg = config.to_c()
        ctx = C.c_void_p()
        L.check(self._lib.aeth_galore_create(C.byref(self._cfg), specs, len(param_specs), self.device, C.byref(ctx)),
                "aeth_galore_create")
        self._ctx = ctx
        self._pending_deltas: dict = {}
        self._info: dict = {}
        for i, spec in enumerate(param_specs):
            info = L.ParamInfo()
            L.check(self._lib.aeth_galore_param_info(self._ctx, i, C.byref(info)))
            self._info[(spec[0], spec[1])] = (i, info)

    def close(self):
        if getattr(self, "_ctx", None):
            self._lib.aeth_galore_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    # ---- helpers ----
    def _key(self, layer_idx, param_name):
        return self._info.get((layer_idx, param_name))

    def param_info(self, layer_idx, param_name) -> L.ParamInfo | None:
        k = self._key(layer_idx, param_name)
        return None if k is None else k[1]

    def index(self, layer_idx, param_name) -> int:
        k = self._key(layer_idx, param_name)
        return -1 if k is None else k[0]

    # ---- OptimizerBackend (doublepass/src/lib.rs:62-107) ----
    def project_and_accumulate(self, grad: torch.Tensor, layer_idx: int, param_name: str) -> None:
        """optimizer.rs:264-292; wrong-sized gradients and unknown keys are ignored."""
        k = self._key(layer_idx, param_name)
        if k is None:
            return
        idx, info = k
        if grad.numel() != info.m * info.n:
            return
        g = grad.contiguous()
        L.check(self._lib.aeth_galore_project_accumulate(self._ctx, idx, _ptr(g), _DTYPES[g.dtype],
                                                         C.c_void_p(_stream_handle())), "project_and_accumulate")

    def lowrank_grad_sqnorm(self, layer_idx: int, param_name: str) -> float:
        """optimizer.rs:294-301 (0.0 for unknown keys)."""
        k = self._key(layer_idx, param_name)
        if k is None:
            return 0.0
        out = C.c_double()
        L.check(self._lib.aeth_galore_sqnorm(self._ctx, k[0], C.byref(out), C.c_void_p(_stream_handle())),
                "lowrank_grad_sqnorm")
        return out.value

    def apply_update(self, layer_idx: int, param_name: str, clip_scale: float, weight=None,
                     prequant_out: torch.Tensor | None = None) -> None:
        """optimizer.rs:303-362.  Without `weight` the delta (lr applied) is
        kept for take_weight_delta, as the reference does.  With `weight` (an
        fp32 tensor or an NF4Tensor) the update is applied in place."""
        k = self._key(layer_idx, param_name)
        if k is None:
            return
        idx, info = k
        w = L.WeightRef()
        delta = None
        if weight is None:
            delta = torch.empty(info.m, info.n, dtype=torch.float32, device=f"cuda:{self.device}")
            w.kind, w.delta_out = L.WEIGHT_NONE, delta.data_ptr()
        elif isinstance(weight, NF4Tensor):
            w.kind, w.data, w.absmax = L.WEIGHT_NF4, weight.packed.data_ptr(), weight.absmax.data_ptr()
        else:
            w.kind, w.data = L.WEIGHT_F32, weight.data_ptr()
        if prequant_out is not None:
            w.prequant_out = prequant_out.data_ptr()
        L.check(self._lib.aeth_galore_apply_update(self._ctx, idx, float(clip_scale), None, C.byref(w),
                                                   C.c_void_p(_stream_handle())), "apply_update")
        if delta is not None:
            self._pending_deltas[(layer_idx, param_name)] = delta

    def zero_accum(self, layer_idx: int, param_name: str) -> None:
        k = self._key(layer_idx, param_name)
        if k is not None:
            L.check(self._lib.aeth_galore_zero_accum(self._ctx, k[0], C.c_void_p(_stream_handle())), "zero_accum")

    def notify_step(self, step: int) -> None:
        """Records the step and runs pending subspace refreshes (optimizer.rs:373-398)
        on the current stream."""
        L.check(self._lib.aeth_galore_notify_step_async(self._ctx, step, C.c_void_p(_stream_handle())),
                "notify_step")

    def optimizer_version(self) -> int:
        """Completed subspace refreshes (optimizer.rs:249-253)."""
        return int(self._lib.aeth_galore_version(self._ctx))

    def save_state(self, path) -> None:
        """flush_all_to_file (optimizer.rs:180-192) to `path`: the reference's
        version 2 layout in REF mode, version 3 in B200 mode."""
        L.check(self._lib.aeth_galore_save_state(self._ctx, str(path).encode(), C.c_void_p(_stream_handle())),
                "save_state")

    def load_state(self, path) -> None:
        """The state part of GaLoreOptimizer::open (optimizer.rs:135-176): projectors,
        INT8 m/v and scales, step count and Adam constants from `path`."""
        L.check(self._lib.aeth_galore_load_state(self._ctx, str(path).encode(), C.c_void_p(_stream_handle())),
                "load_state")

    def projector_kind(self, layer_idx: int, param_name: str) -> ProjectorKind:
        return ProjectorKind.ORTHONORMAL

    def true_frobenius_sqnorm(self, layer_idx: int, param_name: str):
        return None

    # ---- GaLoreOptimizer inherent methods ----
    def take_weight_delta(self, layer_idx: int, param_name: str):
        """optimizer.rs:195-200"""
        return self._pending_deltas.pop((layer_idx, param_name), None)

    def step_count(self) -> int:
        return int(self._lib.aeth_galore_step_count(self._ctx))

    # ---- state access (tests, checkpointing) ----
    def get_projector(self, layer_idx, param_name):
        idx, info = self._key(layer_idx, param_name)
        dev = f"cuda:{self.device}"
        if info.side == 0:
            P = torch.empty(info.m, info.rank, device=dev)
            Q = torch.empty(info.n, info.rank, device=dev)
        else:
            s = info.m if info.side == 1 else info.n
            P = torch.empty(s, info.rank, device=dev) if info.side == 1 else None
            Q = torch.empty(s, info.rank, device=dev) if info.side == 2 else None
        L.check(self._lib.aeth_galore_get_projector(self._ctx, idx, _ptr(P), _ptr(Q), C.c_void_p(_stream_handle())))
        return P, Q

    def set_projector(self, layer_idx, param_name, P=None, Q=None):
        idx, _ = self._key(layer_idx, param_name)
        P = None if P is None else P.contiguous().float()
        Q = None if Q is None else Q.contiguous().float()
        L.check(self._lib.aeth_galore_set_projector(self._ctx, idx, _ptr(P), _ptr(Q), C.c_void_p(_stream_handle())),
                "set_projector")

    def get_state(self, layer_idx, param_name):
        idx, info = self._key(layer_idx, param_name)
        dev = f"cuda:{self.device}"
        m8 = torch.empty(info.state_elems, dtype=torch.int8, device=dev)
        v8 = torch.empty_like(m8)
        ms = torch.empty(info.state_blocks, dtype=torch.float32, device=dev)
        vs = torch.empty_like(ms)
        L.check(self._lib.aeth_galore_get_state(self._ctx, idx, _ptr(m8), _ptr(v8), _ptr(ms), _ptr(vs),
                                                C.c_void_p(_stream_handle())))
        return m8, v8, ms, vs

    def set_state(self, layer_idx, param_name, m8, v8, ms, vs):
        idx, _ = self._key(layer_idx, param_name)
        L.check(self._lib.aeth_galore_set_state(self._ctx, idx, _ptr(m8), _ptr(v8), _ptr(ms), _ptr(vs),
                                                C.c_void_p(_stream_handle())))

    def get_accum(self, layer_idx, param_name):
        idx, info = self._key(layer_idx, param_name)
        out = torch.empty(info.state_elems, dtype=torch.float32, device=f"cuda:{self.device}")
        L.check(self._lib.aeth_galore_get_accum(self._ctx, idx, _ptr(out), C.c_void_p(_stream_handle())))
        return out

    # ---- fused whole-layer step (device-side deferred_apply_with_clip) ----
    def _indices(self, keys):
        return (C.c_int * len(keys))(*[self._key(*k)[0] for k in keys])

    @staticmethod
    def _weight_refs(weights, prequant_outs=None):
        if weights is None:
            return None
        wrefs = (L.WeightRef * len(weights))()
        for i, w in enumerate(weights):
            if isinstance(w, NF4Tensor):
                wrefs[i].kind, wrefs[i].data, wrefs[i].absmax = L.WEIGHT_NF4, w.packed.data_ptr(), w.absmax.data_ptr()
            elif w is None:
                wrefs[i].kind = L.WEIGHT_NONE
            else:
                wrefs[i].kind, wrefs[i].data = L.WEIGHT_F32, w.data_ptr()
            if prequant_outs is not None and prequant_outs[i] is not None:
                wrefs[i].prequant_out = prequant_outs[i].data_ptr()
        return wrefs

    def _hook(self, sq_hook):
        if sq_hook is None:
            return L.SQ_HOOK(0)

        def _cb(sq_ptr, count, stream, user):  # noqa: ARG001 - C callback signature
            try:
                sq_hook(_wrap_device_doubles(sq_ptr, count, self.device))
                return 0
            except Exception:  # noqa: BLE001 - reported as a status to C
                return L.AETH_ERR_CONFIG
        return L.SQ_HOOK(_cb)

    def step_layer(self, keys, grads, weights=None, sq_hook=None):
        """project_and_accumulate for every (layer, name) in `keys`, the exact
        global-norm clip on the device, then apply_update + zero_accum
        (hook.rs:139-203) -- no host synchronisation.  `sq_hook(sq_tensor)`
        may all-reduce the per-parameter squared norms (multi-GPU).  Returns
        the device clip coefficient (a 1-element tensor)."""
        n = len(keys)
        gp = (C.c_void_p * n)(*[g.data_ptr() for g in grads])
        clip = torch.empty(1, dtype=torch.float32, device=f"cuda:{self.device}")
        hook = self._hook(sq_hook)
        L.check(self._lib.aeth_galore_step(self._ctx, n, self._indices(keys), gp, _DTYPES[grads[0].dtype],
                                           self._weight_refs(weights), hook, None, _ptr(clip),
                                           C.c_void_p(_stream_handle())), "aeth_galore_step")
        return clip

    def project_layer(self, keys, grads):
        """project_and_accumulate for the (layer, name) keys of one layer, in
        grouped launches, as backward.rs:509-521 calls it when the layer's
        gradients are ready; the gradient buffers may be refilled once this
        work has run on the current stream."""
        n = len(keys)
        gp = (C.c_void_p * n)(*[g.data_ptr() for g in grads])
        L.check(self._lib.aeth_galore_project_layer(self._ctx, n, self._indices(keys), gp, _DTYPES[grads[0].dtype],
                                                    C.c_void_p(_stream_handle())), "aeth_galore_project_layer")

    def refresh_layer(self, keys, grads):
        """The streamed subspace refresh (B200 mode): new projectors for these
        parameters from this step's gradients, by the tensor-core randomized
        SVD, installed (with an Adam state reset) by the next notify_step."""
        n = len(keys)
        gp = (C.c_void_p * n)(*[g.data_ptr() for g in grads])
        L.check(self._lib.aeth_galore_refresh_layer(self._ctx, n, self._indices(keys), gp, _DTYPES[grads[0].dtype],
                                                    C.c_void_p(_stream_handle())), "aeth_galore_refresh_layer")

    def refresh_due(self) -> bool:
        """Whether the step in progress is a refresh step: step + 1 == 1 or a
        multiple of switch_interval (optimizer.rs:264-292)."""
        nxt = self.step_count() + 1
        every = self.config.switch_interval
        return nxt == 1 or (every > 0 and nxt % every == 0)

    def projector_buffer(self, layer_idx, param_name) -> torch.Tensor:
        """The bf16 projector of a B200 parameter's side as a torch view of the
        optimizer's own buffer (s x rank), for broadcasting it; read-only."""
        idx, _ = self._key(layer_idx, param_name)
        ptr_ = C.c_void_p()
        rows, cols = C.c_int(), C.c_int()
        L.check(self._lib.aeth_galore_projector_buffer(self._ctx, idx, C.byref(ptr_), C.byref(rows), C.byref(cols)),
                "aeth_galore_projector_buffer")
        return _wrap_device(int(ptr_.value), (rows.value, cols.value), "<i2", self.device).view(torch.bfloat16)

    def finish_step(self, keys, weights=None, sq_hook=None, clip_out: torch.Tensor | None = None,
                    prequant_outs=None):
        """The exact global-norm clip over every listed parameter (all that this
        GPU owns) in one launch, then Adam and the weight write for all of them
        (hook.rs:115-203 on the device).  Returns the device clip coefficient.
        `prequant_outs` (optional, one fp32 tensor or None per weight) receive
        the updated weights before NF4 requantisation."""
        n = len(keys)
        clip = clip_out if clip_out is not None else torch.empty(1, dtype=torch.float32,
                                                                 device=f"cuda:{self.device}")
        hook = self._hook(sq_hook)
        L.check(self._lib.aeth_galore_finish_step(self._ctx, n, self._indices(keys),
                                                  self._weight_refs(weights, prequant_outs), hook, None, _ptr(clip),
                                                  C.c_void_p(_stream_handle())), "aeth_galore_finish_step")
        return clip

    # ---- per-phase device timing of step_layer ----
    PHASES = ("projection", "sqnorm_clip", "adam", "apply")

    def set_phase_timing(self, enable: bool) -> None:
        L.check(self._lib.aeth_galore_set_phase_timing(self._ctx, 1 if enable else 0), "set_phase_timing")

    def phase_times(self):
        """(steps, {phase: total device ms}) over the step_layer, project_layer and
        finish_step calls since the last call (steps counts step_layer and
        finish_step calls)."""
        out = (C.c_double * 4)()
        steps = C.c_int(0)
        L.check(self._lib.aeth_galore_phase_times(self._ctx, out, C.byref(steps)), "phase_times")
        return steps.value, dict(zip(self.PHASES, list(out)))

    # ---- global clip over several GPUs through peer memory ----
    def clip_handle(self, world: int) -> bytes:
        """Allocates this optimizer's clip slots for a group of `world` GPUs and
        returns their CUDA IPC handle (64 bytes) for the other ranks."""
        buf = C.create_string_buffer(L.CLIP_HANDLE_BYTES)
        L.check(self._lib.aeth_galore_clip_handle(self._ctx, world, buf), "clip_handle")
        return buf.raw

    def set_clip_group(self, rank: int, world: int, handles, timeout_s: float = 2.0) -> None:
        """Joins the clip group: `handles` lists every rank's clip_handle() in
        rank order.  All ranks must meet at a barrier after this call and
        then call step_layer equally often, without sq_hook."""
        blob = b"".join(handles) if world > 1 else b""
        if world > 1 and len(blob) != world * L.CLIP_HANDLE_BYTES:
            raise ValueError("set_clip_group: one 64-byte handle per rank expected")
        buf = C.create_string_buffer(blob, max(len(blob), 1))
        L.check(self._lib.aeth_galore_set_clip_group(self._ctx, rank, world, buf, int(timeout_s * 1e9)),
                "set_clip_group")

    def set_clip_group_ptrs(self, rank: int, slots, timeout_s: float = 2.0) -> None:
        """Joins a clip group whose slot pointers the caller mapped itself
        (`slots[rank]` must be clip_slots())."""
        arr = (C.c_void_p * len(slots))(*slots)
        L.check(self._lib.aeth_galore_set_clip_group_ptrs(self._ctx, rank, len(slots), arr, int(timeout_s * 1e9)),
                "set_clip_group_ptrs")

    def clip_slots(self) -> int:
        """Device address of this optimizer's clip slots (after clip_handle)."""
        p = C.c_void_p()
        L.check(self._lib.aeth_galore_clip_slots(self._ctx, C.byref(p)), "clip_slots")
        return int(p.value)


def _wrap_device(ptr: int, shape, typestr: str, device: int) -> torch.Tensor:
    """A torch view of device memory owned by the library (no copy)."""
    class _Holder:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                             "version": 2, "strides": None}
    with torch.cuda.device(device):
        return torch.as_tensor(_Holder(), device=f"cuda:{device}")


def _wrap_device_doubles(ptr: int, count: int, device: int) -> torch.Tensor:
    """A torch view of `count` device doubles owned by the library (no copy)."""
    return _wrap_device(ptr, (count,), "<f8", device)


@dataclass
class ClipResult:
    """doublepass/src/hook.rs:70-94"""
    global_grad_norm: float
    clip_coeff: float
    clipped: bool
    used_grouped_fallback: bool
    frobenius_exact_layers: int


def _f32(x: float) -> float:
    import numpy as np
    return float(np.float32(x))


def deferred_apply_with_clip(optimizer, max_grad_norm: float, trainable_layers) -> ClipResult:
    """doublepass/src/hook.rs:115-136 (global clip, grouped fallback for ProjectorKind.NONE)."""
    if not trainable_layers:
        raise ValueError("deferred_apply_with_clip: trainable_layers must not be empty")
    if any(optimizer.projector_kind(li, pn) == ProjectorKind.NONE for li, pn in trainable_layers):
        return _grouped_clip_fallback(optimizer, max_grad_norm, trainable_layers)
    gsq = 0.0
    exact = 0
    for li, pn in trainable_layers:
        kind = optimizer.projector_kind(li, pn)
        if kind == ProjectorKind.RANDOM:
            fsq = optimizer.true_frobenius_sqnorm(li, pn)
            if fsq is not None:
                exact += 1
                gsq += fsq
                continue
        gsq += optimizer.lowrank_grad_sqnorm(li, pn)
    gnorm = gsq ** 0.5
    clip = min(_f32(max_norm_f64(max_grad_norm) / (gnorm + 1e-6)), 1.0)
    for li, pn in trainable_layers:
        optimizer.apply_update(li, pn, clip)
        optimizer.zero_accum(li, pn)
    return ClipResult(gnorm, clip, clip < 1.0, False, exact)


def max_norm_f64(x: float) -> float:
    """TrainingPlan::max_grad_norm is an f32 widened to f64 (hook.rs:144)."""
    return _f32(x)


def _grouped_clip_fallback(optimizer, max_grad_norm, trainable_layers) -> ClipResult:
    """doublepass/src/hook.rs:214-259"""
    layers: dict = {}
    for li, pn in trainable_layers:
        layers.setdefault(li, []).append(pn)
    total = 0.0
    min_clip = 1.0
    for li in sorted(layers):
        sq = sum(optimizer.lowrank_grad_sqnorm(li, pn) for pn in layers[li])
        clip = min(_f32(max_norm_f64(max_grad_norm) / (sq ** 0.5 + 1e-6)), 1.0)
        for pn in layers[li]:
            optimizer.apply_update(li, pn, clip)
            optimizer.zero_accum(li, pn)
        total += sq
        min_clip = min(min_clip, clip)
    return ClipResult(total ** 0.5, min_clip, min_clip < 1.0, True, 0)
