"""Op implementations (same module layout and names as the reference's triton_ops.kernels)."""

from triton_ops.kernels.fp8_gemm import FP8Linear, fp8_gemm, fp8_gemm_kernel
from triton_ops.kernels.fp8_quantize import (
    dequantize_fp8,
    dequantize_fp8_kernel,
    quantize_fp8,
    quantize_fp8_kernel,
)
from triton_ops.kernels.gated_mlp import FusedGatedMLP, fused_gated_mlp, fused_gated_mlp_kernel
from triton_ops.kernels.rmsnorm_rope import (
    FusedRMSNormRoPE,
    fused_rmsnorm_rope,
    fused_rmsnorm_rope_kernel,
    rmsnorm_kernel,
    rope_kernel,
)

__all__ = [
    "fused_rmsnorm_rope",
    "FusedRMSNormRoPE",
    "rmsnorm_kernel",
    "rope_kernel",
    "fused_rmsnorm_rope_kernel",
    "fused_gated_mlp",
    "FusedGatedMLP",
    "fused_gated_mlp_kernel",
    "fp8_gemm",
    "FP8Linear",
    "fp8_gemm_kernel",
    "quantize_fp8",
    "dequantize_fp8",
    "quantize_fp8_kernel",
    "dequantize_fp8_kernel",
]
