"""The C-ABI library loads without a GPU and exports every symbol its header declares."""

import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "tfo_b200.h"


def header_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TFO_API\s+[\w\s\*]+?\b(tfo_\w+)\s*\(", text)))


def test_header_declares_the_hot_path():
    syms = header_symbols()
    for name in ("tfo_rmsnorm_rope", "tfo_fp8_quantize", "tfo_fp8_dequantize", "tfo_fp8_compute_scale",
                 "tfo_fp8_gemm", "tfo_gated_mlp", "tfo_last_error", "tfo_device_error_flags"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from triton_ops import _lib

    lib = _lib.load()
    for name in header_symbols():
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"
    # and the Python binding declares exactly the header's entry points
    assert sorted(_lib.declared_symbols()) == header_symbols()


def test_library_is_sm100a_only_and_self_contained():
    from triton_ops import _lib

    path = _lib.LIB_PATH
    assert path.exists()
    data = path.read_bytes()
    assert b"sm_100a" in data or b"sm_100" in data


def test_version_and_error_strings():
    from triton_ops import _lib

    assert "sm_100a" in _lib.version()
    lib = _lib.load()
    # argument errors are reported without touching a GPU
    st = lib.tfo_fp8_quantize(None, 16, 7, None, None, None, 3, None, 0, None)
    assert st == _lib.ERR_DTYPE
    assert b"f16, bf16 or f32" in lib.tfo_last_error()
    st = lib.tfo_rmsnorm_rope(None, None, None, None, None, 1, 1, 64, 63, 1, 64, 1, 1e-6, 0, 0, 0, 0, None)
    assert st == _lib.ERR_INVALID
    assert b"even" in lib.tfo_last_error()
    st = lib.tfo_fp8_gemm(None, None, None, None, None, 4, 4, 200000, 3, 0, 0, None, 0, None)
    assert st == _lib.ERR_INVALID


def test_empty_problems_are_no_ops_without_a_gpu():
    from triton_ops import _lib

    lib = _lib.load()
    assert lib.tfo_rmsnorm_rope(None, None, None, None, None, 0, 5, 64, 64, 1, 64, 1, 1e-6, 0, 0, 0, 0, None) == 0
    assert lib.tfo_fp8_dequantize(None, 0, 3, None, None, 0, None) == 0
    assert lib.tfo_gated_mlp(None, None, None, None, 0, 8, 8, 0, 0, 0, None, 0, None) == 0


def test_workspace_queries():
    from triton_ops import _lib

    lib = _lib.load()
    assert lib.tfo_fp8_gemm_workspace_bytes(128, 256, 100, 3, 0) >= 128 * 112 + 256 * 112
    assert lib.tfo_gated_mlp_workspace_bytes(64, 64, 64, 0, 0) == 0  # fp16 x fp16: no copies
    assert lib.tfo_gated_mlp_workspace_bytes(64, 64, 64, 0, 2) >= 64 * 64 * 4  # fp16 x with fp32 weights


def test_extension_loads_and_declines_what_it_does_not_serve():
    """The PyTorch extension is built in-tree, links the same library, and returns None
    (so that the Python wrapper validates and raises) for inputs outside its common case."""
    import torch

    from triton_ops import _lib

    ext = _lib.ext()
    assert ext is not None, "build the extension with triton-fused-ops_b200/build.py"
    for name in ("quantize_dynamic", "linear_prepared", "clear_workspaces"):
        assert hasattr(ext, name)
    assert ext.quantize_dynamic(torch.zeros(4), _lib.U8) is None  # CPU tensor
    w = torch.zeros(8, 16, dtype=torch.int8)
    assert ext.linear_prepared(torch.zeros(2, 16), w, torch.zeros(8, dtype=torch.int32), torch.ones(()), None) is None
    _lib.clear_workspaces()


def test_extension_errors_map_to_package_exceptions():
    import pytest

    from triton_ops import _lib
    from triton_ops.exceptions import TritonKernelError, UnsupportedDtypeError

    with pytest.raises(UnsupportedDtypeError):
        _lib.raise_ext_error(RuntimeError("tfo status 2: tfo_fp8_quantize: x must be f16, bf16 or f32"))
    with pytest.raises(TritonKernelError, match="status 3"):
        _lib.raise_ext_error(RuntimeError("tfo status 3: tfo_fp8_quantize: out of memory"))
