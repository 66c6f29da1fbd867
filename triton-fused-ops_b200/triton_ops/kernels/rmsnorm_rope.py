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
