"""Host-side logic that needs no GPU: validation, exceptions, models, tile table, compat classes."""

import pytest
import torch

import triton_ops
from triton_ops.exceptions import (
    DeviceError,
    NumericalOverflowError,
    ShapeMismatchError,
    TritonKernelError,
    UnsupportedDtypeError,
)


def test_public_api_matches_reference_names():
    for name in ["fused_rmsnorm_rope", "FusedRMSNormRoPE", "fused_gated_mlp", "FusedGatedMLP", "fp8_gemm",
                 "FP8Linear", "quantize_fp8", "dequantize_fp8", "TensorSpec", "RMSNormRoPEInput", "GatedMLPInput",
                 "FP8GEMMInput", "KernelMetrics", "TuningResult", "FP8Format", "TritonKernelError",
                 "ShapeMismatchError", "UnsupportedDtypeError", "NumericalOverflowError", "TuningFailedError",
                 "TritonAutoTuner", "ConfigCache", "RMSNORM_ROPE_CONFIGS", "GATED_MLP_CONFIGS",
                 "FP8_GEMM_CONFIGS", "BenchmarkSuite", "CorrectnessVerifier", "PerformanceReport"]:
        assert hasattr(triton_ops, name), name
    from triton_ops import api
    from triton_ops.kernels import (  # noqa: F401
        dequantize_fp8_kernel,
        fp8_gemm_kernel,
        fused_gated_mlp_kernel,
        fused_rmsnorm_rope_kernel,
        quantize_fp8_kernel,
        rmsnorm_kernel,
        rope_kernel,
    )
    from triton_ops.kernels.fp8_gemm import fp8_gemm_reference  # noqa: F401
    from triton_ops.kernels.fp8_quantize import quantize_fp8_with_overflow_handling  # noqa: F401
    from triton_ops.kernels.gated_mlp import gated_mlp_reference  # noqa: F401
    from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope_reference  # noqa: F401

    assert set(api.__all__) >= {"fused_rmsnorm_rope", "fused_gated_mlp", "fp8_gemm", "quantize_fp8",
                                "dequantize_fp8"}


def test_native_kernel_handles_are_not_triton_launchable():
    from triton_ops.kernels import fp8_gemm_kernel

    with pytest.raises(TypeError):
        fp8_gemm_kernel[(1,)]


def test_cpu_tensors_raise_device_error_no_fallback():
    x = torch.randn(2, 4, 64, dtype=torch.float16)
    w = torch.ones(64, dtype=torch.float16)
    cs = torch.randn(4, 64, dtype=torch.float16)
    with pytest.raises(DeviceError):
        triton_ops.fused_rmsnorm_rope(x, w, cs, cs)
    with pytest.raises(DeviceError):
        triton_ops.fused_gated_mlp(x, torch.randn(32, 64).half(), torch.randn(32, 64).half())
    with pytest.raises(DeviceError):
        triton_ops.quantize_fp8(x)
    with pytest.raises(DeviceError):
        triton_ops.fp8_gemm(torch.randn(4, 8).half(), torch.randn(8, 4).half())
    with pytest.raises(DeviceError):
        triton_ops.dequantize_fp8(torch.zeros(4, dtype=torch.uint8), torch.tensor(1.0))
    with pytest.raises(DeviceError):
        triton_ops.FP8Format.compute_scale(x)


def test_exception_hierarchy_and_attributes():
    e = ShapeMismatchError("m", expected=(2, 16, 256), actual=(2, 16, 128), tensor_name="x")
    assert (e.expected, e.actual, e.tensor_name) == ((2, 16, 256), (2, 16, 128), "x")
    e = NumericalOverflowError("o", max_value=1000.0, scale=0.5, attempts=3)
    assert (e.max_value, e.scale, e.attempts) == (1000.0, 0.5, 3)
    e = DeviceError("d", expected_device="cuda", actual_device="cpu", tensor_name="w")
    assert e.actual_device == "cpu"
    for cls in (ShapeMismatchError, UnsupportedDtypeError, NumericalOverflowError, DeviceError):
        assert issubclass(cls, TritonKernelError)


def test_models():
    from triton_ops.models import FP8GEMMInput, GatedMLPInput, KernelMetrics, RMSNormRoPEInput, TensorSpec

    spec = TensorSpec(shape=(2, 16, 256), dtype=torch.float16, device="cpu")
    assert spec.validate(torch.randn(2, 16, 256).half())
    assert not spec.validate(torch.randn(2, 16, 128).half())
    assert not spec.validate(torch.randn(2, 16, 256))
    assert RMSNormRoPEInput.from_shapes(2, 16, 256, 64).cos.shape == (16, 64)
    assert GatedMLPInput.from_shapes(2, 16, 256, 512).gate_weight.shape == (512, 256)
    assert FP8GEMMInput.from_shapes(8, 16, 32).b.shape == (32, 16)
    s = str(KernelMetrics(latency_ms=1.5, throughput_tflops=10.0, bandwidth_gbps=1000.0, bandwidth_utilization=50.0))
    assert "1.5" in s and "10" in s and "1000" in s and "50" in s


def test_tile_table_rules():
    from triton_ops.autotuner import tile_table as tt

    assert tt.fp8_gemm_config(8192, 4096, 4096)["BLOCK_N"] == 256
    assert tt.fp8_gemm_config(8192, 4096, 4096)["CTAS_PER_MMA"] == 2
    assert tt.fp8_gemm_config(16, 4096, 4096)["BLOCK_N"] == 128
    assert tt.fp8_gemm_config(16, 4096, 4096)["SPLIT_K"] == 4
    assert tt.fp8_gemm_config(4096, 96, 4096)["BLOCK_N"] == 128
    c = tt.rmsnorm_rope_config(4096, 64)
    assert c["kernel"] == 1 and c["threads"] == 256 and c["vectors"] == 2
    assert tt.rmsnorm_rope_config(4096, 64, rows=65536)["kernel"] == 2
    assert tt.rmsnorm_rope_config(4100, 64)["kernel"] == 0  # rows not a whole number of 16-byte vectors
    assert tt.rmsnorm_rope_config(4096, 48)["kernel"] == 0  # 48/8 = 6 vectors per head: generic path
    assert tt.gated_mlp_config(2048, 11264, 4096)["BLOCK_M"] == 256


def test_tile_table_matches_library():
    """The Python statement of the launch table equals the library's own choice (tfo_select_tile)."""
    import os

    from triton_ops import _lib
    from triton_ops.autotuner import tile_table as tt

    pair = os.environ.get("TFO_B200_PAIR_MMA", "1") != "0"
    keys = ("BLOCK_M", "BLOCK_N", "CTAS_PER_MMA", "STAGES", "SPLIT_K", "GROUP_M")
    for M in (1, 16, 100, 128, 129, 256, 1000, 1024, 4096, 8192, 65536):
        for N in (64, 128, 129, 1000, 4096, 11264, 40000):
            for K in (16, 128, 512, 4096):
                want = [tt.fp8_gemm_config(M, N, K, pair=pair)[k] for k in keys]
                assert _lib.select_tile(_lib.OP_FP8_GEMM, M, N, K, _lib.U8) == want, (M, N, K)
                want = [tt.gated_mlp_config(M, N, K, pair=pair)[k] for k in keys]
                assert _lib.select_tile(_lib.OP_GATED_MLP, M, N, K, _lib.F16) == want, (M, N, K)
    rk = ("kernel", "threads", "vectors", "full", "smem")
    for rows in (1, 256, 4096, 8192, 65536):
        for hidden, hd in ((4096, 64), (4096, 128), (2048, 64), (1024, 32), (8192, 128), (4096, 48), (4100, 50),
                           (5120, 128), (16384, 128)):
            for code, eb in ((_lib.F16, 2), (_lib.BF16, 2), (_lib.F32, 4)):
                want = [tt.rmsnorm_rope_config(hidden, hd, eb, rows=rows)[k] for k in rk] + [0]
                assert _lib.select_tile(_lib.OP_RMSNORM_ROPE, rows, hidden, hd, code) == want, (rows, hidden, hd, eb)


def test_autotuner_and_cache_roundtrip(tmp_path):
    from triton_ops import ConfigCache, TritonAutoTuner

    calls = []

    def fn(x, BLOCK=1):
        calls.append(BLOCK)
        return x * BLOCK

    tuner = TritonAutoTuner(fn, {"BLOCK": [1, 2, 4]}, warmup_runs=1, benchmark_runs=2, cache_dir=str(tmp_path))
    res = tuner.tune(3, problem_size=(1, 2), device="cpu", kernel_type="toy")
    assert res.best_config["BLOCK"] in (1, 2, 4)
    assert tuner.get_cached_config((1, 2), "cpu", "toy") == res.best_config
    cache2 = ConfigCache(str(tmp_path))
    assert ("toy", (1, 2), "cpu") in cache2 and len(cache2) == 1
    cache2.clear()
    assert len(cache2) == 0


def test_correctness_verifier():
    from triton_ops import CorrectnessVerifier

    v = CorrectnessVerifier(rtol=1e-3, atol=1e-5)
    a = torch.ones(10)
    ok, det = v.verify(a, a + 1e-7)
    assert ok and det["num_violations"] == 0
    ok, det = v.verify(a, a * 2)
    assert not ok and det["num_violations"] == 10
    assert v.compute_relative_error(a, a) == 0.0


def test_validation_order_matches_reference_on_cpu():
    from triton_ops.validation import validate_gated_mlp_inputs

    x = torch.randn(2, 4, 8)
    # device is checked before the activation name, as in the reference
    with pytest.raises(DeviceError):
        validate_gated_mlp_inputs(x, torch.randn(4, 8), torch.randn(4, 8), activation="invalid")


def test_workspace_cache_is_bounded_and_clearable(monkeypatch):
    """One buffer per (device, stream), grow-only, least recently used dropped past the cap."""
    from triton_ops import _lib

    handles = iter(range(1000, 2000))
    current = {"h": next(handles)}
    monkeypatch.setattr(_lib, "_raw_stream", lambda idx: current["h"])
    monkeypatch.setattr(_lib, "_is_capturing", lambda: False)
    _lib.clear_workspaces()
    dev = torch.device("cpu", 0)
    a = _lib.workspace(100, dev)
    assert _lib.workspace(50, dev) is a  # same stream, fits: reused
    b = _lib.workspace(1000, dev)
    assert b is not a and b.numel() >= 1000  # grown
    first = current["h"]
    for _ in range(_lib._WS_MAX_ENTRIES + 3):  # a new stream per call
        current["h"] = next(handles)
        _lib.workspace(16, dev)
    assert len(_lib._ws_cache) == _lib._WS_MAX_ENTRIES
    assert (0, first) not in _lib._ws_cache  # the oldest stream's buffer was dropped
    _lib.clear_workspaces()
    assert len(_lib._ws_cache) == 0
