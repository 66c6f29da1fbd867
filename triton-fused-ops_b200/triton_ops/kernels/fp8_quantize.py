"""Per-tensor FP8 quantization / dequantization.

``quantize_fp8`` returns the reference's 8-bit code (a ``uint8`` tensor,
``u = int8(rint(clamp(x*s, +-448) / 448 * 127)) + 128``) bit-exactly, plus the
0-dim fp32 scale ``s = 448 / max|x|`` (reference:
triton_ops/kernels/fp8_quantize.py:128-173, 258-287). The scale is computed on
the GPU (no ``.item()`` host sync) and equals the reference's host value bit
for bit. Passing ``dtype=torch.float8_e4m3fn`` instead produces true e4m3
bytes of ``clamp(x*s, +-448)``.

``dequantize_fp8`` inverts either encoding: ``out = dec(q) / s``
(reference: :176-211, oracle :290-312).

Both also accept a scale with one value per row of the last dimension
(shape ``[..., 1]``: per-token activations, per-output-channel ``[out, in]``
weights), an extension: the reference's kernels read a single scale.

The ``*_reference`` functions are plain-PyTorch restatements of the
reference's oracles, kept importable for tests; the ops never call them.
"""

from __future__ import annotations

import torch

from triton_ops import _lib
from triton_ops.exceptions import NumericalOverflowError, UnsupportedDtypeError
from triton_ops.kernels._native import NativeKernel
from triton_ops.models import FP8Format
from triton_ops.validation import SUPPORTED_DTYPES_FLOAT, _check_cuda, validate_fp8_quantize_inputs

FP8_MAX = 448.0
FP8_MIN_NORMAL = 2**-6

quantize_fp8_kernel = NativeKernel("quantize_fp8_kernel", "tfo_fp8_quantize", "amax -> scale -> 8-bit encode")
dequantize_fp8_kernel = NativeKernel("dequantize_fp8_kernel", "tfo_fp8_dequantize", "8-bit decode via 256-entry table")
compute_scale_kernel = NativeKernel("compute_scale_kernel", "tfo_fp8_compute_scale", "grid-wide amax -> scale")

_CODE_DTYPES = (torch.uint8,) + ((torch.float8_e4m3fn,) if hasattr(torch, "float8_e4m3fn") else ())
_QCODE = {torch.uint8: _lib.U8, **({torch.float8_e4m3fn: _lib.E4M3} if hasattr(torch, "float8_e4m3fn") else {})}


def _row_scales(tensor: torch.Tensor, scale: torch.Tensor):
    """The per-row scale vector (fp32, contiguous) if `scale` holds one value per row of
    `tensor` viewed as [numel / last_dim, last_dim] (shape [..., 1] or [rows]); else None."""
    if scale is None or scale.numel() <= 1 or tensor.dim() < 1:
        return None
    cols = tensor.shape[-1]
    rows = tensor.numel() // max(cols, 1)
    if scale.numel() != rows or (scale.dim() == tensor.dim() and scale.shape[-1] != 1):
        raise ValueError(f"a scale tensor must hold one value per row ({rows}) of the last dimension, "
                         f"got shape {tuple(scale.shape)}")
    return scale.to(device=tensor.device, dtype=torch.float32).reshape(rows).contiguous()


def _scale_f32(scale: torch.Tensor) -> torch.Tensor:
    """The first element of `scale` as a contiguous fp32 device tensor (what the kernels read)."""
    if scale.dtype == torch.float32 and scale.is_contiguous():
        return scale
    return scale.reshape(-1)[:1].to(torch.float32).contiguous()


def quantize_fp8(
    tensor: torch.Tensor,
    scale: torch.Tensor = None,
    *,
    dtype: torch.dtype = torch.uint8,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize a float tensor to 8 bits with a per-tensor scale.

    Args:
        tensor: fp16 / bf16 / fp32 CUDA tensor (contiguous)
        scale: optional multiplier; when None it is computed as 448 / max|x|
        dtype: ``torch.uint8`` (default: the reference's code) or
            ``torch.float8_e4m3fn``

    Returns:
        (codes shaped like `tensor`, scale) — the scale is the tensor passed in,
        or a new 0-dim fp32 CUDA tensor.
    """
    if scale is None:
        fast = _lib.ext()
        if fast is not None:
            # one C++ call for the common case (CUDA, contiguous, float input, known code dtype)
            try:
                r = fast.quantize_dynamic(tensor, _QCODE.get(dtype, -1))
            except RuntimeError as exc:
                _lib.raise_ext_error(exc)
            if r is not None:
                return r
    validate_fp8_quantize_inputs(tensor, scale)
    if dtype not in _CODE_DTYPES:
        raise UnsupportedDtypeError(
            f"quantize_fp8 output dtype must be one of {_CODE_DTYPES}, got {dtype}",
            dtype=dtype, supported_dtypes=list(_CODE_DTYPES),
        )
    dev = tensor.device
    out = torch.empty(tensor.shape, dtype=dtype, device=dev)
    n = tensor.numel()
    x_code = _lib.dtype_code(tensor.dtype, "tensor")
    out_code = _lib.dtype_code(dtype)
    stream = _lib.stream_of(tensor)
    if scale is None:
        scale = torch.empty((), dtype=torch.float32, device=dev)
        ws_bytes = _lib.load().tfo_fp8_scale_workspace_bytes(n)
        ws = _lib.workspace(ws_bytes, dev)
        _lib.call("tfo_fp8_quantize", tensor.data_ptr(), n, x_code, None, scale.data_ptr(), out.data_ptr(),
                  out_code, ws.data_ptr(), ws.numel(), stream)
        return out, scale
    if scale.device != dev:
        scale = scale.to(dev)
    rs = _row_scales(tensor, scale)
    if rs is not None:
        # per-token / per-channel scales: one multiplier per row of the last dimension
        if n:
            _lib.call("tfo_fp8_quantize_rows", tensor.data_ptr(), rs.numel(), tensor.shape[-1], x_code, rs.data_ptr(),
                      out.data_ptr(), out_code, stream)
        return out, scale
    s32 = _scale_f32(scale)
    if n:
        _lib.call("tfo_fp8_quantize", tensor.data_ptr(), n, x_code, s32.data_ptr(), None, out.data_ptr(),
                  out_code, None, 0, stream)
    return out, scale


def quantize_fp8_per_token(
    tensor: torch.Tensor,
    *,
    dtype: torch.dtype = torch.uint8,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize with one dynamic scale per row of the last dimension (per token).

    Returns ``(codes, scales)`` equal byte for byte to
    ``scales = FP8Format.compute_scale_per_channel(tensor, dim=-1)`` followed by
    ``codes, _ = quantize_fp8(tensor, scales, dtype=dtype)``: ``scales`` has
    shape ``[..., 1]`` and `tensor`'s dtype. One kernel computes each row's
    max, its scale and its codes, reading `tensor` once from memory, where the
    two calls read it twice in three launches. An extension: the reference
    quantizes with a single scale.
    """
    _check_cuda(tensor, "tensor")
    if tensor.dtype not in SUPPORTED_DTYPES_FLOAT:
        raise UnsupportedDtypeError(
            f"quantize_fp8_per_token input dtype must be one of {SUPPORTED_DTYPES_FLOAT}, got {tensor.dtype}",
            dtype=tensor.dtype, supported_dtypes=list(SUPPORTED_DTYPES_FLOAT),
        )
    if dtype not in _CODE_DTYPES:
        raise UnsupportedDtypeError(
            f"quantize_fp8_per_token output dtype must be one of {_CODE_DTYPES}, got {dtype}",
            dtype=dtype, supported_dtypes=list(_CODE_DTYPES),
        )
    if tensor.dim() < 1:
        raise ValueError("quantize_fp8_per_token needs a tensor with at least one dimension")
    x = tensor.contiguous()
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    scales = torch.empty(*x.shape[:-1], 1, dtype=x.dtype, device=x.device)
    if rows and cols:
        _lib.call("tfo_fp8_quantize_per_token", x.data_ptr(), rows, cols, _lib.dtype_code(x.dtype, "tensor"),
                  scales.data_ptr(), out.data_ptr(), _lib.dtype_code(dtype), _lib.stream_of(x))
    return out, scales


def dequantize_fp8(
    tensor: torch.Tensor,
    scale: torch.Tensor,
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """Decode 8-bit codes (``uint8`` reference code or ``float8_e4m3fn``): ``dec(q) / scale``."""
    _check_cuda(tensor, "tensor")
    _check_cuda(scale, "scale")
    if tensor.dtype not in _CODE_DTYPES:
        raise UnsupportedDtypeError(
            f"dequantize_fp8 expects uint8 or float8_e4m3fn codes, got {tensor.dtype}",
            dtype=tensor.dtype, supported_dtypes=list(_CODE_DTYPES), tensor_name="tensor",
        )
    if output_dtype not in SUPPORTED_DTYPES_FLOAT:
        raise UnsupportedDtypeError(
            f"output_dtype must be float16, bfloat16 or float32, got {output_dtype}",
            dtype=output_dtype, supported_dtypes=list(SUPPORTED_DTYPES_FLOAT),
        )
    out = torch.empty(tensor.shape, dtype=output_dtype, device=tensor.device)
    q = tensor.contiguous()
    n = q.numel()
    if n:
        rs = _row_scales(q, scale)
        if rs is not None:
            _lib.call("tfo_fp8_dequantize_rows", q.data_ptr(), rs.numel(), q.shape[-1], _lib.dtype_code(q.dtype),
                      rs.data_ptr(), out.data_ptr(), _lib.dtype_code(output_dtype), _lib.stream_of(q))
            return out
        s32 = _scale_f32(scale.to(tensor.device))
        _lib.call("tfo_fp8_dequantize", q.data_ptr(), n, _lib.dtype_code(q.dtype), s32.data_ptr(), out.data_ptr(),
                  _lib.dtype_code(output_dtype), _lib.stream_of(q))
    return out


def quantize_fp8_with_overflow_handling(
    tensor: torch.Tensor,
    scale: torch.Tensor = None,
    max_attempts: int = 3,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize, halving the scale (up to `max_attempts` + 1 checks) while x*scale leaves +-448.

    Same control flow as the reference (fp8_quantize.py:214-255); raises
    NumericalOverflowError when no tried scale keeps the tensor in range.
    """
    if scale is None:
        scale = FP8Format.compute_scale(tensor)
    for _ in range(max_attempts):
        if FP8Format.is_in_range(tensor, scale):
            return quantize_fp8(tensor, scale)
        scale = scale / 2.0
    if FP8Format.is_in_range(tensor, scale):
        return quantize_fp8(tensor, scale)
    raise NumericalOverflowError(
        f"Cannot quantize tensor to FP8 after {max_attempts} attempts",
        max_value=tensor.abs().max().item(),
        scale=scale.item() if scale.numel() == 1 else None,
        attempts=max_attempts,
    )


def fp8_quantize_reference(tensor: torch.Tensor, scale: torch.Tensor = None) -> tuple[torch.Tensor, torch.Tensor]:
    """PyTorch restatement of the reference's quantize oracle (uint8 codes, scale)."""
    if scale is None:
        max_abs = tensor.abs().max()
        if max_abs == 0:
            scale = torch.tensor(1.0, device=tensor.device, dtype=torch.float32)
        else:
            scale = torch.tensor(FP8_MAX / max_abs.item(), device=tensor.device, dtype=torch.float32)
    clamped = torch.clamp(tensor.float() * scale, -FP8_MAX, FP8_MAX)
    codes = torch.round(clamped / FP8_MAX * 127.0).to(torch.int8) + 128
    return codes.to(torch.uint8), scale


def fp8_dequantize_reference(
    tensor: torch.Tensor, scale: torch.Tensor, output_dtype: torch.dtype = torch.float16
) -> torch.Tensor:
    """PyTorch restatement of the reference's dequantize oracle."""
    values = (tensor.to(torch.int32) - 128).float() / 127.0 * FP8_MAX
    return (values / scale).to(output_dtype)
