"""Fused RMSNorm + rotary position embedding (rotate-half convention).

``fused_rmsnorm_rope`` launches the sm_100a kernel behind ``tfo_rmsnorm_rope``
(csrc/rmsnorm_rope.cu): one pass per token row, RMS reduction, weight, and the
per-head rotation with ``cos/sin[pos, :head_dim/2]``, ``pos = row % seq_len``.
Drop-in for the reference's triton_ops/kernels/rmsnorm_rope.py:238-302.

The ``*_reference`` functions are plain-PyTorch restatements of the
reference's test oracles (rmsnorm_rope.py:305-383). They exist so code and
tests written against the reference keep importing them; the op never calls
them.
"""

from __future__ import annotations

import torch

from triton_ops import _lib
from triton_ops.kernels._native import NativeKernel
from triton_ops.validation import check_rmsnorm_rope_kernel_bounds, validate_rmsnorm_rope_inputs

fused_rmsnorm_rope_kernel = NativeKernel(
    "fused_rmsnorm_rope_kernel", "tfo_rmsnorm_rope", "one-pass RMSNorm + rotate-half RoPE per token row"
)
# The reference also exports unfused halves that it never launches; both map
# to the fused entry point here.
rmsnorm_kernel = NativeKernel("rmsnorm_kernel", "tfo_rmsnorm_rope", "RMSNorm (fused with RoPE here)")
rope_kernel = NativeKernel("rope_kernel", "tfo_rmsnorm_rope", "RoPE (fused with RMSNorm here)")
fused_rmsnorm_rope_quantize_kernel = NativeKernel(
    "fused_rmsnorm_rope_quantize_kernel", "tfo_rmsnorm_rope_quantize", "RMSNorm + RoPE rows with amax partials -> 8-bit encode"
)


def fused_rmsnorm_rope(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float = 1e-6,
    num_heads: int = None,
) -> torch.Tensor:
    """RMSNorm over the hidden dim, then rotate-half RoPE on each head.

    Args:
        x: [batch, seq_len, hidden_dim], fp16 / bf16 / fp32, contiguous
        weight: [hidden_dim] RMSNorm weight (any float dtype)
        cos, sin: [seq_len, head_dim] or [1, seq_len, 1, head_dim]; only the
            first head_dim/2 columns are read
        eps: added to mean(x^2) before the square root
        num_heads: heads to rotate (default hidden_dim // head_dim); columns
            past num_heads * head_dim are normalised but not rotated

    Returns:
        A new tensor shaped and typed like x.
    """
    batch_size, seq_len, hidden_dim, head_dim, num_heads = validate_rmsnorm_rope_inputs(x, weight, cos, sin, num_heads)
    check_rmsnorm_rope_kernel_bounds(x, cos, sin, seq_len, hidden_dim, head_dim, num_heads)
    if weight.device != x.device:
        from triton_ops.exceptions import DeviceError

        raise DeviceError("weight must be on x's device", expected_device=str(x.device),
                          actual_device=str(weight.device), tensor_name="weight")
    if cos.dim() == 4:
        cos = cos.squeeze(0).squeeze(1)
        sin = sin.squeeze(0).squeeze(1)
    if sin.stride() != cos.stride():
        cos = cos.contiguous()
        sin = sin.contiguous()

    out = torch.empty_like(x)
    if out.numel() == 0:
        return out
    _lib.call(
        "tfo_rmsnorm_rope",
        x.data_ptr(), weight.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(),
        batch_size, seq_len, hidden_dim, head_dim, num_heads,
        cos.stride(0), cos.stride(1), float(eps),
        _lib.dtype_code(x.dtype, "x"), _lib.dtype_code(weight.dtype, "weight"),
        _lib.dtype_code(cos.dtype, "cos"), _lib.dtype_code(sin.dtype, "sin"),
        _lib.stream_of(x),
    )
    return out


def fused_rmsnorm_rope_quantize(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float = 1e-6,
    num_heads: int = None,
    scale: torch.Tensor = None,
    *,
    dtype: torch.dtype = torch.uint8,
) -> tuple:
    """RMSNorm + RoPE with the output quantized to 8 bits in the same kernel.

    Returns ``(codes, scale)`` equal, byte for byte, to
    ``quantize_fp8(fused_rmsnorm_rope(x, weight, cos, sin, eps, num_heads), scale, dtype=dtype)``.
    With ``scale=None`` the dynamic per-tensor scale is derived from maxima the
    RMSNorm+RoPE pass records while it writes the rows (on shapes where it
    runs its warp-per-row kernel), so the encode pass needs no separate amax
    read of the rows. This is the fusion the reference's roadmap pairs with
    ``FP8Linear`` (a ``FusedRMSNormRoPE`` -> ``FP8Linear`` chain); the
    reference itself has no such op.

    Args:
        x, weight, cos, sin, eps, num_heads: as for :func:`fused_rmsnorm_rope`
        scale: optional quantize multiplier (tensor); None = dynamic per-tensor scale
        dtype: ``torch.uint8`` (the reference's code) or ``torch.float8_e4m3fn``
    """
    from triton_ops.exceptions import UnsupportedDtypeError
    from triton_ops.kernels.fp8_quantize import _CODE_DTYPES, _scale_f32

    batch_size, seq_len, hidden_dim, head_dim, num_heads = validate_rmsnorm_rope_inputs(x, weight, cos, sin, num_heads)
    check_rmsnorm_rope_kernel_bounds(x, cos, sin, seq_len, hidden_dim, head_dim, num_heads)
    if dtype not in _CODE_DTYPES:
        raise UnsupportedDtypeError(f"codes dtype must be one of {_CODE_DTYPES}, got {dtype}", dtype=dtype,
                                    supported_dtypes=list(_CODE_DTYPES))
    if weight.device != x.device:
        from triton_ops.exceptions import DeviceError

        raise DeviceError("weight must be on x's device", expected_device=str(x.device),
                          actual_device=str(weight.device), tensor_name="weight")
    if cos.dim() == 4:
        cos = cos.squeeze(0).squeeze(1)
        sin = sin.squeeze(0).squeeze(1)
    if sin.stride() != cos.stride():
        cos = cos.contiguous()
        sin = sin.contiguous()
    dev = x.device
    codes = torch.empty(x.shape, dtype=dtype, device=dev)
    x_code = _lib.dtype_code(x.dtype, "x")
    s32 = None
    scale_out = None
    if scale is None:
        scale = scale_out = torch.empty((), dtype=torch.float32, device=dev)
    else:
        s32 = _scale_f32(scale.to(dev))
    lib = _lib.load()
    ws_bytes = lib.tfo_rmsnorm_rope_quantize_workspace_bytes(batch_size, seq_len, hidden_dim, x_code)
    ws = _lib.workspace(ws_bytes, dev)
    _lib.call(
        "tfo_rmsnorm_rope_quantize",
        x.data_ptr(), weight.data_ptr(), cos.data_ptr(), sin.data_ptr(), codes.data_ptr(),
        batch_size, seq_len, hidden_dim, head_dim, num_heads, cos.stride(0), cos.stride(1), float(eps),
        x_code, _lib.dtype_code(weight.dtype, "weight"), _lib.dtype_code(cos.dtype, "cos"),
        _lib.dtype_code(sin.dtype, "sin"), _lib.ptr(s32), _lib.ptr(scale_out), _lib.dtype_code(dtype),
        ws.data_ptr(), ws.numel(), _lib.stream_of(x),
    )
    return codes, scale


def rmsnorm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """PyTorch RMSNorm: ``x / sqrt(mean(x^2) + eps) * weight`` in fp32, cast to x.dtype."""
    xf = x.float()
    rms = torch.sqrt(torch.mean(xf**2, dim=-1, keepdim=True) + eps)
    return (xf / rms * weight.float()).to(x.dtype)


def rope_reference(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """PyTorch rotate-half RoPE over heads of size cos.shape[-1]."""
    batch, seq_len, hidden_dim = x.shape
    head_dim = cos.shape[-1]
    half = head_dim // 2
    heads = x.view(batch, seq_len, hidden_dim // head_dim, head_dim)
    first, second = heads[..., :half].float(), heads[..., half:].float()
    c = cos[:seq_len, :half].float()[None, :, None, :]
    s = sin[:seq_len, :half].float()[None, :, None, :]
    rotated = torch.cat([first * c - second * s, first * s + second * c], dim=-1)
    return rotated.to(x.dtype).view(batch, seq_len, hidden_dim)


def fused_rmsnorm_rope_reference(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float = 1e-6,
) -> torch.Tensor:
    """PyTorch composition RMSNorm -> RoPE (accepts 2-D or 4-D cos/sin)."""
    if cos.dim() == 4:
        cos = cos.squeeze(0).squeeze(1)
        sin = sin.squeeze(0).squeeze(1)
    return rope_reference(rmsnorm_reference(x, weight, eps), cos, sin)


class FusedRMSNormRoPE(torch.nn.Module):
    """Module form: holds the fp32 RMSNorm weight (initialised to ones)."""

    def __init__(self, hidden_dim: int, head_dim: int, eps: float = 1e-6):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.head_dim = head_dim
        self.eps = eps
        self.num_heads = hidden_dim // head_dim
        self.weight = torch.nn.Parameter(torch.ones(hidden_dim))

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        return fused_rmsnorm_rope(x, self.weight, cos, sin, self.eps, self.num_heads)
