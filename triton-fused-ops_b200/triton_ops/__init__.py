"""B200-native fused transformer ops, drop-in for the reference's ``triton_ops``.

Ops (each one launches hand-written sm_100a CUDA kernels through the C ABI in
``include/tfo_b200.h``; there is no Triton and no CPU fallback):

* ``fused_rmsnorm_rope`` / ``FusedRMSNormRoPE``
* ``fused_gated_mlp`` / ``FusedGatedMLP``
* ``fp8_gemm`` / ``FP8Linear``
* ``quantize_fp8`` / ``dequantize_fp8``

Example::

    >>> import torch
    >>> from triton_ops import fused_rmsnorm_rope
    >>> x = torch.randn(2, 128, 4096, device="cuda", dtype=torch.float16)
    >>> w = torch.ones(4096, device="cuda", dtype=torch.float16)
    >>> cos = torch.randn(128, 64, device="cuda", dtype=torch.float16)
    >>> sin = torch.randn(128, 64, device="cuda", dtype=torch.float16)
    >>> y = fused_rmsnorm_rope(x, w, cos, sin)
"""

__version__ = "0.1.0"

from triton_ops.autotuner import (
    FP8_GEMM_CONFIGS,
    GATED_MLP_CONFIGS,
    RMSNORM_ROPE_CONFIGS,
    ConfigCache,
    TritonAutoTuner,
)
from triton_ops.benchmark import BenchmarkSuite, CorrectnessVerifier, PerformanceReport
from triton_ops.exceptions import (
    DeviceError,
    NumericalOverflowError,
    ShapeMismatchError,
    TritonKernelError,
    TuningFailedError,
    UnsupportedDtypeError,
)
from triton_ops.kernels.fp8_gemm import FP8Linear, fp8_gemm
from triton_ops.kernels.fp8_quantize import dequantize_fp8, quantize_fp8, quantize_fp8_per_token
from triton_ops.kernels.gated_mlp import FusedGatedMLP, fused_gated_mlp, fused_gated_mlp_quantize
from triton_ops.kernels.rmsnorm_rope import FusedRMSNormRoPE, fused_rmsnorm_rope, fused_rmsnorm_rope_quantize
from triton_ops.models import (
    FP8Format,
    FP8GEMMInput,
    GatedMLPInput,
    KernelMetrics,
    RMSNormRoPEInput,
    TensorSpec,
    TuningResult,
)

__all__ = [
    "fused_rmsnorm_rope",
    "fused_rmsnorm_rope_quantize",
    "FusedRMSNormRoPE",
    "fused_gated_mlp",
    "fused_gated_mlp_quantize",
    "FusedGatedMLP",
    "fp8_gemm",
    "FP8Linear",
    "quantize_fp8",
    "quantize_fp8_per_token",
    "dequantize_fp8",
    "TensorSpec",
    "RMSNormRoPEInput",
    "GatedMLPInput",
    "FP8GEMMInput",
    "KernelMetrics",
    "TuningResult",
    "FP8Format",
    "TritonKernelError",
    "ShapeMismatchError",
    "UnsupportedDtypeError",
    "NumericalOverflowError",
    "TuningFailedError",
    "DeviceError",
    "TritonAutoTuner",
    "ConfigCache",
    "RMSNORM_ROPE_CONFIGS",
    "GATED_MLP_CONFIGS",
    "FP8_GEMM_CONFIGS",
    "BenchmarkSuite",
    "CorrectnessVerifier",
    "PerformanceReport",
]
