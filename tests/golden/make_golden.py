"""Generate NF4 golden fixtures by running the reference's own quantiser.

Run in a container that has the reference checkout (it is not needed, and not
present, where the tests run):

    python tests/golden/make_golden.py /path/to/reference

It imports ``aethelStream/shard_engine/python/pipeline/quantizer.py`` by file
path (the package ``__init__`` pulls in ``accelerate``, which this image lacks)
and records, for a set of seeded inputs, the reference's packed nibbles, fp32
absmax and fp16 dequantised output.  ``nf4_golden.npz`` is the committed
result; ``tests/test_oracle_golden.py`` pins the C oracle against it.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch


def load_quantizer(ref_root: str):
    path = os.path.join(ref_root, "aethelStream", "shard_engine", "python", "pipeline", "quantizer.py")
    spec = importlib.util.spec_from_file_location("ref_nf4_quantizer", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_nf4_quantizer"] = mod
    spec.loader.exec_module(mod)
    return mod


def cases():
    g = torch.Generator().manual_seed(0)
    out = {}
    # shard_engine/tests/test_nf4_fidelity.py:8-9 input (randn 256x256 fp16, seed 42).
    torch.manual_seed(42)
    out["fidelity_256x256_f16"] = torch.randn(256, 256, dtype=torch.float16)
    out["zeros_64x64"] = torch.zeros(64, 64)
    # the weight distribution of the benchmark configs: N(0, 0.02)
    out["w_n002_64x512"] = torch.randn(64, 512, generator=g) * 0.02
    # ragged sizes: partial last block (quantizer pads with zeros)
    out["ragged_200"] = torch.randn(200, generator=g)
    out["ragged_130"] = torch.randn(130, generator=g) * 3.0
    # extreme and tiny magnitudes (the 1e-8 clamp path)
    out["scaled_1000_32x64"] = torch.randn(32, 64, generator=g) * 1000.0
    out["tiny_1e-9_128"] = torch.randn(128, generator=g) * 1e-9
    # values placed on the decision boundaries between adjacent codes
    codes = torch.tensor([-1.0, -0.6961928, -0.52507305, -0.3949175, -0.28444138, -0.18477343, -0.09105004, 0.0,
                          0.0795803, 0.1609302, 0.2461123, 0.33791524, 0.44070983, 0.562617, 0.72295684, 1.0])
    mids = (codes[:-1] + codes[1:]) / 2.0
    blk = torch.cat([torch.tensor([1.0]), mids, -mids, mids * 0.5, torch.zeros(64 - 1 - 15 * 3)])
    nudged = torch.cat([torch.tensor([1.0]), torch.nextafter(mids, torch.full_like(mids, 2.0)),
                        torch.nextafter(mids, torch.full_like(mids, -2.0)), torch.zeros(64 - 1 - 30)])
    out["boundaries_128"] = torch.cat([blk, nudged])
    # Student-t like heavy tails (the 13B config's gradient distribution)
    t = torch.distributions.StudentT(3.0).sample((4096,))
    out["studentt_4096"] = t.float() * 1e-3
    # non-finite values: a NaN makes the block's absmax NaN (all codes 0); an
    # infinite absmax sends finite values to code 7 and +-inf to code 0
    nf = torch.randn(320, generator=g) * 0.02
    nf[3] = float("nan")
    nf[70] = float("inf")
    nf[140] = float("-inf")
    nf[141] = float("inf")
    nf[200] = float("nan")
    nf[201] = float("-inf")
    out["nonfinite_320"] = nf
    return out


def main(ref_root: str):
    qz = load_quantizer(ref_root)
    arrays = {}
    for name, x in cases().items():
        res = qz.quantize_nf4(x)
        arrays[f"{name}__input"] = x.float().numpy().ravel()
        arrays[f"{name}__packed"] = res.packed.numpy().astype(np.uint8)
        arrays[f"{name}__absmax"] = res.absmax.numpy().astype(np.float32)
        try:
            deq = qz.dequantize_nf4(res)
            arrays[f"{name}__deq_f16"] = deq.numpy().ravel().astype(np.float16)
        except RuntimeError:
            pass  # dequantize_nf4 reshapes by block count; some ragged sizes do not divide
    here = os.path.dirname(os.path.abspath(__file__))
    np.savez_compressed(os.path.join(here, "nf4_golden.npz"), **arrays)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    torch.manual_seed(0)
    # the reference checkout: first argument, else $AETH_REFERENCE_ROOT
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETH_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set AETH_REFERENCE_ROOT)")
    main(root)
