"""The C-ABI library: loads without a GPU, exports every symbol the header
declares, and its host-only entry points behave as specified."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "aeth_galore.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"(?m)^\s*(?:int|void|const char\*|uint64_t)\s+\*?(\w+)\s*\(", text)
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__
    __graft_entry__.build()  # loads aethelstream_b200/build.py by path, then the package
    from aethelstream_b200 import _lib as L
    return L


def test_header_declares_reference_symbols():
    names = header_functions()
    for ref_symbol in ("galore_project_forward", "galore_project_backward", "galore_quantize_absmax_f32_to_i8",
                       "galore_dequantize_i8_to_f32", "doublepass_galore_apply"):
        assert ref_symbol in names


def test_library_exports_every_header_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    missing = [n for n in header_functions() if n not in exported]
    assert not missing, missing


def test_binding_covers_header(lib):
    assert sorted(lib.SIGNATURES) == header_functions()


def test_import_fails_loudly_without_library(lib, tmp_path):
    with pytest.raises(ImportError):
        lib.load(str(tmp_path / "libaeth_galore.so"))


def test_config_defaults_mirror_reference(lib):
    """GaLoreConfig / AdamWConfig / LayerRankConfig / TrainingPlan defaults
    (optimizer.rs:49-60, adamw.rs:23-33, layer_rank.rs:19-27, plan.rs)."""
    c = lib.GaloreConfig()
    lib.load().aeth_galore_config_default(C.byref(c))
    assert (c.default_rank, c.attn_rank, c.mlp_rank, c.vector_rank) == (16, 32, 16, 8)
    assert (c.switch_interval, c.oversampling) == (200, 10)
    assert np.float32(c.beta1) == np.float32(0.9) and np.float32(c.beta2) == np.float32(0.999)
    assert np.float32(c.eps) == np.float32(1e-8) and np.float32(c.lr) == np.float32(1e-3)
    assert c.weight_decay == 0.0 and c.scale_lr_by_rank == 0 and c.max_grad_norm == 1.0
    assert c.state_codec == lib.CODEC_PER_TENSOR and c.state_block == 2048


@pytest.mark.parametrize("signed", [True, False])
def test_dynamic_map_matches_oracle(lib, oracle, signed):
    out = (C.c_float * 256)()
    assert lib.load().aeth_dynamic_map(int(signed), out) == 0
    mine = np.frombuffer(out, np.float32).copy()
    ref = oracle.dynamic_map(signed)
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))
    assert np.all(np.diff(mine) > 0)
    assert mine[-1] == 1.0 and 0.0 in mine
    if not signed:
        assert mine[0] == 0.0


def test_argument_errors_need_no_gpu(lib):
    """Bad dimensions return the reference's -1 before any device work
    (galore_project.cu:74,123; quantize_state.cu:67,94)."""
    L = lib.load()
    assert L.galore_project_forward(None, None, None, None, None, 0, 4, 4, None) == -1
    assert L.galore_project_backward(None, None, None, None, None, 4, -1, 4, None) == -1
    assert L.galore_quantize_absmax_f32_to_i8(None, None, None, 0, None) == -1
    assert L.galore_dequantize_i8_to_f32(None, None, 1.0, 0, None) == -1
    assert L.aeth_nf4_dequant(None, None, 0, 64, None, 0, None) == -1
    L.doublepass_galore_apply(None, None, None, None, 1.0, 0.9, 0.999, 1e-8, 1e-3, 0, 1)
    assert L.aeth_last_error() == -1


def test_status_strings(lib):
    L = lib.load()
    assert L.aeth_status_string(0) == b"ok"
    assert L.aeth_status_string(-6) == b"device wait timed out"
    assert b"sm_100a" in L.aeth_version()
