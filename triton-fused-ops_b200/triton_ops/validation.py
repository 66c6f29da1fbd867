"""Host-side argument checks for the ops.

Function names, argument order, return values and the exception raised for
each failure follow the reference (triton_ops/validation.py:24-348), so its
tests and callers see the same behaviour:

* tensor not on CUDA            -> DeviceError
* dtype outside the allowed set -> UnsupportedDtypeError
* non-contiguous input          -> ValueError
* incompatible shapes           -> ShapeMismatchError
* unknown activation            -> ValueError

Checks the reference lacks but that guard the native kernels against
out-of-bounds reads (odd head_dim, num_heads * head_dim > hidden, a 4-D RoPE
table shorter than seq_len, tensors on different GPUs) raise
ShapeMismatchError / DeviceError as well.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from triton_ops.exceptions import DeviceError, ShapeMismatchError, UnsupportedDtypeError

SUPPORTED_DTYPES_FLOAT = [torch.float16, torch.bfloat16, torch.float32]
SUPPORTED_DTYPES_FP8 = [torch.uint8]
if hasattr(torch, "float8_e4m3fn"):
    SUPPORTED_DTYPES_FP8.append(torch.float8_e4m3fn)
if hasattr(torch, "float8_e5m2"):
    SUPPORTED_DTYPES_FP8.append(torch.float8_e5m2)

ACTIVATIONS = ("silu", "gelu", "gelu_tanh")


def _check_cuda(tensor: torch.Tensor, tensor_name: str) -> None:
    if not tensor.is_cuda:
        raise DeviceError(
            f"{tensor_name} must be on CUDA device, got {tensor.device}",
            expected_device="cuda",
            actual_device=str(tensor.device),
            tensor_name=tensor_name,
        )


def _check_same_device(ref: torch.Tensor, tensor: torch.Tensor, tensor_name: str) -> None:
    if tensor.device != ref.device:
        raise DeviceError(
            f"{tensor_name} is on {tensor.device} but the op runs on {ref.device}",
            expected_device=str(ref.device),
            actual_device=str(tensor.device),
            tensor_name=tensor_name,
        )


def _check_dtype(tensor: torch.Tensor, tensor_name: str, supported_dtypes: List[torch.dtype]) -> None:
    if tensor.dtype not in supported_dtypes:
        raise UnsupportedDtypeError(
            f"{tensor_name} has unsupported dtype {tensor.dtype}, supported: {supported_dtypes}",
            dtype=tensor.dtype,
            supported_dtypes=supported_dtypes,
            tensor_name=tensor_name,
        )


def _check_contiguous(tensor: torch.Tensor, tensor_name: str) -> None:
    if not tensor.is_contiguous():
        raise ValueError(f"{tensor_name} must be contiguous")


def validate_rmsnorm_rope_inputs(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_heads: Optional[int] = None,
) -> Tuple[int, int, int, int, int]:
    """Checks fused RMSNorm+RoPE inputs.

    x is [batch, seq_len, hidden], weight [hidden], cos/sin [seq_len, head_dim]
    or [1, seq_len, 1, head_dim]. Returns (batch, seq_len, hidden, head_dim,
    num_heads); num_heads defaults to hidden // head_dim.
    """
    for t, n in ((x, "x"), (weight, "weight"), (cos, "cos"), (sin, "sin")):
        _check_cuda(t, n)
    for t, n in ((x, "x"), (weight, "weight"), (cos, "cos"), (sin, "sin")):
        _check_dtype(t, n, SUPPORTED_DTYPES_FLOAT)
    _check_contiguous(x, "x")
    _check_contiguous(weight, "weight")

    if x.dim() != 3:
        raise ShapeMismatchError(
            f"x must be 3D [batch, seq_len, hidden_dim], got {x.dim()}D",
            expected=(None, None, None),
            actual=x.shape,
            tensor_name="x",
        )
    batch_size, seq_len, hidden_dim = x.shape

    if weight.shape != (hidden_dim,):
        raise ShapeMismatchError(
            f"weight shape {weight.shape} doesn't match hidden_dim {hidden_dim}",
            expected=(hidden_dim,),
            actual=weight.shape,
            tensor_name="weight",
        )

    if cos.dim() == 2:
        if cos.shape[0] != seq_len:
            raise ShapeMismatchError(
                f"cos seq_len {cos.shape[0]} doesn't match x seq_len {seq_len}",
                expected=(seq_len, None),
                actual=cos.shape,
                tensor_name="cos",
            )
        head_dim = cos.shape[1]
    elif cos.dim() == 4:
        head_dim = cos.shape[3]
    else:
        raise ShapeMismatchError(f"cos must be 2D or 4D, got {cos.dim()}D", tensor_name="cos")

    if sin.shape != cos.shape:
        raise ShapeMismatchError(
            f"sin shape {sin.shape} doesn't match cos shape {cos.shape}",
            expected=cos.shape,
            actual=sin.shape,
            tensor_name="sin",
        )

    if num_heads is None:
        if head_dim == 0 or hidden_dim % head_dim != 0:
            raise ShapeMismatchError(
                f"hidden_dim {hidden_dim} must be divisible by head_dim {head_dim}",
                tensor_name="x",
            )
        num_heads = hidden_dim // head_dim

    return batch_size, seq_len, hidden_dim, head_dim, num_heads


def check_rmsnorm_rope_kernel_bounds(
    x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, seq_len: int, hidden: int, head_dim: int, num_heads: int
) -> None:
    """Extra checks that keep every kernel access inside the given tensors."""
    for t, n in ((cos, "cos"), (sin, "sin")):
        _check_same_device(x, t, n)
    if head_dim <= 0 or head_dim % 2 != 0:
        raise ShapeMismatchError(f"head_dim must be even and positive, got {head_dim}", tensor_name="cos")
    if num_heads < 0 or num_heads * head_dim > hidden:
        raise ShapeMismatchError(
            f"num_heads {num_heads} x head_dim {head_dim} exceeds hidden_dim {hidden}", tensor_name="x"
        )
    if cos.dim() == 4:
        if cos.shape[0] != 1 or cos.shape[2] != 1 or cos.shape[1] < seq_len:
            raise ShapeMismatchError(
                f"4-D cos/sin must be [1, >=seq_len, 1, head_dim], got {tuple(cos.shape)}",
                expected=(1, seq_len, 1, head_dim),
                actual=cos.shape,
                tensor_name="cos",
            )


def validate_gated_mlp_inputs(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    activation: str = "silu",
) -> Tuple[int, int, int, int]:
    """Checks gated-MLP inputs; returns (batch, seq_len, hidden, intermediate).

    Accepted activations: "silu", "gelu" (erf form) and "gelu_tanh".
    """
    for t, n in ((x, "x"), (gate_weight, "gate_weight"), (up_weight, "up_weight")):
        _check_cuda(t, n)
    for t, n in ((x, "x"), (gate_weight, "gate_weight"), (up_weight, "up_weight")):
        _check_dtype(t, n, SUPPORTED_DTYPES_FLOAT)
    for t, n in ((x, "x"), (gate_weight, "gate_weight"), (up_weight, "up_weight")):
        _check_contiguous(t, n)

    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be 'silu' or 'gelu' (or 'gelu_tanh'), got '{activation}'")

    if x.dim() != 3:
        raise ShapeMismatchError(f"x must be 3D [batch, seq_len, hidden_dim], got {x.dim()}D", tensor_name="x")
    batch_size, seq_len, hidden_dim = x.shape

    if gate_weight.dim() != 2:
        raise ShapeMismatchError(
            f"gate_weight must be 2D [intermediate_dim, hidden_dim], got {gate_weight.dim()}D",
            tensor_name="gate_weight",
        )
    intermediate_dim, gate_hidden = gate_weight.shape
    if gate_hidden != hidden_dim:
        raise ShapeMismatchError(
            f"gate_weight hidden_dim {gate_hidden} doesn't match x hidden_dim {hidden_dim}",
            expected=(None, hidden_dim),
            actual=gate_weight.shape,
            tensor_name="gate_weight",
        )
    if up_weight.shape != gate_weight.shape:
        raise ShapeMismatchError(
            f"up_weight shape {up_weight.shape} doesn't match gate_weight shape {gate_weight.shape}",
            expected=gate_weight.shape,
            actual=up_weight.shape,
            tensor_name="up_weight",
        )
    _check_same_device(x, gate_weight, "gate_weight")
    _check_same_device(x, up_weight, "up_weight")
    return batch_size, seq_len, hidden_dim, intermediate_dim


def validate_fp8_gemm_inputs(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: torch.Tensor,
    b_scale: torch.Tensor,
    output_dtype: torch.dtype = torch.float16,
) -> Tuple[int, int, int]:
    """Checks FP8 GEMM inputs (a [M, K], b [K, N]); returns (M, N, K)."""
    _check_cuda(a, "a")
    _check_cuda(b, "b")
    if a_scale is None or b_scale is None:
        raise ValueError("a_scale and b_scale are required for pre-quantized FP8 operands")
    _check_cuda(a_scale, "a_scale")
    _check_cuda(b_scale, "b_scale")
    _check_contiguous(a, "a")
    _check_contiguous(b, "b")

    if output_dtype not in SUPPORTED_DTYPES_FLOAT:
        raise UnsupportedDtypeError(
            f"output_dtype must be float16, bfloat16, or float32, got {output_dtype}",
            dtype=output_dtype,
            supported_dtypes=list(SUPPORTED_DTYPES_FLOAT),
        )
    if a.dim() != 2:
        raise ShapeMismatchError(f"a must be 2D [M, K], got {a.dim()}D", tensor_name="a")
    if b.dim() != 2:
        raise ShapeMismatchError(f"b must be 2D [K, N], got {b.dim()}D", tensor_name="b")
    M, K_a = a.shape
    K_b, N = b.shape
    if K_a != K_b:
        raise ShapeMismatchError(
            f"Matrix dimensions don't match: a is [{M}, {K_a}], b is [{K_b}, {N}]",
            tensor_name="a, b",
        )
    return M, N, K_a


def validate_fp8_quantize_inputs(tensor: torch.Tensor, scale: Optional[torch.Tensor] = None) -> None:
    """Checks a tensor to be quantized (and its optional scale)."""
    _check_cuda(tensor, "tensor")
    _check_dtype(tensor, "tensor", SUPPORTED_DTYPES_FLOAT)
    _check_contiguous(tensor, "tensor")
    if scale is not None:
        _check_cuda(scale, "scale")
