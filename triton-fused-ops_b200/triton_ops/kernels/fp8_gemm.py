"""FP8 GEMM and the FP8Linear module.

``fp8_gemm(a, b, a_scale, b_scale)`` computes ``dec(a) @ dec(b) / (sa * sb)``
on tcgen05 tensor cores (``tfo_fp8_gemm``, csrc/fp8_gemm.cu). For the
reference's 8-bit code (``uint8`` operands) the product is an exact int8 GEMM
with int32 accumulation; ``float8_e4m3fn`` operands use the FP8 tensor-core
path with fp32 accumulation. Float operands are quantized first, as in the
reference (triton_ops/kernels/fp8_gemm.py:123-187).

``FP8Linear`` keeps the reference's parameters and buffers
(fp8_gemm.py:228-310) but hands the [out, in] code matrix to the GEMM as is
(no per-call transpose) and adds the bias in the GEMM's epilogue
(``tfo_fp8_linear``), with the reference's rounding and dtype promotion.

``fp8_gemm_reference`` restates the reference's PyTorch oracle (:190-225) for
tests; the op never calls it.
"""

from __future__ import annotations

import torch

from triton_ops import _lib
from triton_ops.exceptions import UnsupportedDtypeError
from triton_ops.kernels._native import NativeKernel
from triton_ops.kernels.fp8_quantize import _scale_f32, quantize_fp8
from triton_ops.validation import SUPPORTED_DTYPES_FLOAT, validate_fp8_gemm_inputs

FP8_MAX = 448.0

fp8_gemm_kernel = NativeKernel(
    "fp8_gemm_kernel", "tfo_fp8_gemm", "TMA -> smem ring -> tcgen05.mma (kind::i8 / kind::f8f6f4) -> TMEM -> epilogue"
)

_FLOATS = (torch.float16, torch.bfloat16, torch.float32)


def _gemm_codes(a, b, a_scale, b_scale, output_dtype, b_layout):
    """Launches tfo_fp8_gemm on code tensors; b is [K, N] (B_KN) or [N, K] (B_NK)."""
    if a.dtype != b.dtype:
        raise UnsupportedDtypeError(
            f"fp8_gemm operands must share a code dtype, got {a.dtype} and {b.dtype}",
            dtype=(a.dtype, b.dtype), supported_dtypes=[torch.uint8, getattr(torch, "float8_e4m3fn", None)],
        )
    code = _lib.dtype_code(a.dtype, "a")
    if code not in (_lib.U8, _lib.E4M3):
        raise UnsupportedDtypeError(f"fp8_gemm operands must be uint8 or float8_e4m3fn codes, got {a.dtype}",
                                    dtype=a.dtype, tensor_name="a")
    M, K = a.shape
    N = b.shape[1] if b_layout == _lib.B_KN else b.shape[0]
    c = torch.empty(M, N, dtype=output_dtype, device=a.device)
    if c.numel() == 0:
        return c
    if a_scale.numel() > 1 or b_scale.numel() > 1:
        return _gemm_scaled(a, b, a_scale, b_scale, c, M, N, K, code, b_layout, output_dtype)
    sa = _scale_f32(a_scale.to(a.device))
    sb = _scale_f32(b_scale.to(a.device))
    lib = _lib.load()
    ws_bytes = lib.tfo_fp8_gemm_workspace_bytes(M, N, K, code, b_layout)
    ws = _lib.workspace(ws_bytes, a.device)
    _lib.call(
        "tfo_fp8_gemm", a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(), c.data_ptr(), M, N, K, code,
        b_layout, _lib.dtype_code(output_dtype, "output_dtype"), ws.data_ptr(), ws.numel(), _lib.stream_of(a),
    )
    return c


def _gemm_scaled(a, b, a_scale, b_scale, c, M, N, K, code, b_layout, output_dtype):
    """Per-token A scales (M values) and/or per-channel B scales (N values) in the epilogue."""
    dev = a.device
    a_rows = a_scale.numel() > 1
    b_cols = b_scale.numel() > 1
    if a_rows and a_scale.numel() != M:
        raise ValueError(f"a_scale must hold 1 or M={M} values, got {a_scale.numel()}")
    if b_cols and b_scale.numel() != N:
        raise ValueError(f"b_scale must hold 1 or N={N} values, got {b_scale.numel()}")
    sa = a_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    sb = b_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    ws = _lib.workspace(_lib.load().tfo_fp8_gemm_scaled_workspace_bytes(M, N, K, code, b_layout), dev)
    _lib.call(
        "tfo_fp8_gemm_scaled", a.data_ptr(), b.data_ptr(), sa.data_ptr(), int(a_rows), sb.data_ptr(), int(b_cols),
        c.data_ptr(), M, N, K, code, b_layout, _lib.dtype_code(output_dtype, "output_dtype"), ws.data_ptr(),
        ws.numel(), _lib.stream_of(a),
    )
    return c


def _linear_bias(x_codes, w_codes, x_scale, w_scale, bias, gemm_dtype):
    """`fp8_gemm(x, w.t(), output_dtype=gemm_dtype) + bias` with the bias added in the GEMM epilogue.

    The result has torch's promoted dtype of the two operands of the sum, and the
    same values: the product rounded to `gemm_dtype`, plus the bias in fp32.
    """
    M, K = x_codes.shape
    N = w_codes.shape[0]
    res_dtype = torch.promote_types(gemm_dtype, bias.dtype)
    out = torch.empty(M, N, dtype=res_dtype, device=x_codes.device)
    if out.numel() == 0:
        return out
    b = bias.to(x_codes.device).contiguous()
    code = _lib.dtype_code(x_codes.dtype, "x")
    ws = _lib.workspace(_lib.load().tfo_fp8_gemm_workspace_bytes(M, N, K, code, _lib.B_NK), x_codes.device)
    _lib.call(
        "tfo_fp8_linear", x_codes.data_ptr(), w_codes.data_ptr(), _scale_f32(x_scale.to(x_codes.device)).data_ptr(),
        _scale_f32(w_scale.to(x_codes.device)).data_ptr(), b.data_ptr(), _lib.dtype_code(b.dtype, "bias"),
        out.data_ptr(), M, N, K, code, _lib.dtype_code(gemm_dtype), _lib.dtype_code(res_dtype), ws.data_ptr(),
        ws.numel(), _lib.stream_of(x_codes),
    )
    return out


def _linear_prepared(x_codes, w_s8, w_sums, x_scale, w_scale, bias, gemm_dtype):
    """FP8Linear's GEMM (+ bias in the epilogue) on reference-codec codes with the weight prepared once
    (``tfo_fp8_prepare_weight``): the same values as :func:`_linear_bias` / :func:`_gemm_codes`, with no
    per-call operand preparation."""
    M, K = x_codes.shape
    N = w_s8.shape[0]
    res_dtype = gemm_dtype if bias is None else torch.promote_types(gemm_dtype, bias.dtype)
    out = torch.empty(M, N, dtype=res_dtype, device=x_codes.device)
    if out.numel() == 0:
        return out
    dev = x_codes.device

    def on_dev(t):
        return t if t.device == dev else t.to(dev)

    b = None if bias is None else on_dev(bias).contiguous()
    ws = _lib.workspace(_lib.load().tfo_fp8_gemm_workspace_bytes(M, N, K, _lib.U8, _lib.B_NK), dev)
    _lib.call(
        "tfo_fp8_linear_prepared", x_codes.data_ptr(), w_s8.data_ptr(), w_sums.data_ptr(),
        _scale_f32(on_dev(x_scale)).data_ptr(), _scale_f32(on_dev(w_scale)).data_ptr(),
        None if b is None else b.data_ptr(), -1 if b is None else _lib.dtype_code(b.dtype, "bias"), out.data_ptr(),
        M, N, K, _lib.dtype_code(gemm_dtype), _lib.dtype_code(res_dtype), ws.data_ptr(), ws.numel(),
        _lib.stream_of(x_codes),
    )
    return out


def fp8_gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: torch.Tensor = None,
    b_scale: torch.Tensor = None,
    output_dtype: torch.dtype = torch.float16,
    *,
    quant_dtype: torch.dtype = torch.uint8,
) -> torch.Tensor:
    """FP8 matrix product ``a @ b`` of per-tensor-scaled 8-bit operands.

    Args:
        a: [M, K] codes (``uint8`` or ``float8_e4m3fn``) or a float matrix
        b: [K, N] codes or a float matrix
        a_scale, b_scale: the operands' quantize multipliers (required for
            code operands, computed for float operands)
        output_dtype: float16 (default), bfloat16 or float32
        quant_dtype: code dtype used when a float operand is quantized here
            (``torch.uint8`` = the reference's code, or ``torch.float8_e4m3fn``)

    Returns:
        [M, N] tensor of `output_dtype`.
    """
    if a.dtype in _FLOATS:
        a, a_scale = quantize_fp8(a, dtype=quant_dtype)
    if b.dtype in _FLOATS:
        b, b_scale = quantize_fp8(b, dtype=quant_dtype)
    validate_fp8_gemm_inputs(a, b, a_scale, b_scale, output_dtype)
    return _gemm_codes(a, b, a_scale, b_scale, output_dtype, _lib.B_KN)


def fp8_gemm_reference(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: torch.Tensor = None,
    b_scale: torch.Tensor = None,
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """PyTorch restatement of the reference's oracle: decode each code operand, fp32 matmul."""

    def decode(t, s):
        if t.dtype == torch.uint8:
            return (t.to(torch.int32) - 128).float() / 127.0 * FP8_MAX / s
        return t.float()

    return torch.matmul(decode(a, a_scale), decode(b, b_scale)).to(output_dtype)


class FP8Linear(torch.nn.Module):
    """Linear layer whose weight is stored as per-tensor FP8 codes.

    Same parameters and buffers as the reference: ``weight`` (fp32, N(0, 0.02)
    init), optional zero ``bias``, and the ``weight_fp8`` / ``weight_scale``
    buffers filled on the first forward (or by :meth:`quantize_weights`).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_fp8", None)
        self.register_buffer("weight_scale", None)
        self.weight = torch.nn.Parameter(torch.randn(out_features, in_features) * 0.02)
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self._quantized = False
        self._prepared = None  # (key, int8 weight, row sums): the weight's form for tfo_fp8_linear_prepared

    def quantize_weights(self):
        """Quantizes the weight once (reference codec, per-tensor scale)."""
        if not self._quantized:
            weight_fp8, weight_scale = quantize_fp8(self.weight.data)
            self.weight_fp8 = weight_fp8
            self.weight_scale = weight_scale
            self._quantized = True

    def _prepared_weight(self):
        """The weight codes as int8 (u - 128) with their row sums, made once per weight tensor (and again
        only if ``weight_fp8`` is replaced or modified in place)."""
        w = self.weight_fp8
        key = (w.data_ptr(), w._version, w.device)
        if self._prepared is None or self._prepared[0] != key:
            N, K = w.shape
            w_s8 = torch.empty(N, K, dtype=torch.int8, device=w.device)
            sums = torch.empty(N, dtype=torch.int32, device=w.device)
            _lib.call("tfo_fp8_prepare_weight", w.data_ptr(), N, K, w_s8.data_ptr(), sums.data_ptr(),
                      _lib.stream_of(w))
            self._prepared = (key, w_s8, sums)
        return self._prepared[1], self._prepared[2]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        prep = self._prepared
        if prep is not None:
            w = self.weight_fp8
            fast = _lib.ext()
            if fast is not None and prep[0] == (w.data_ptr(), w._version, w.device):
                # the weight is unchanged since it was prepared: quantize x, GEMM and
                # bias in one C++ call (None outside the common case)
                try:
                    out = fast.linear_prepared(x, prep[1], prep[2], self.weight_scale, self.bias)
                except RuntimeError as exc:
                    _lib.raise_ext_error(exc)
                if out is not None:
                    return out
        self.quantize_weights()
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features)
        if not x_2d.is_contiguous():
            x_2d = x_2d.contiguous()
        x_fp8, x_scale = quantize_fp8(x_2d)
        out_dtype = x.dtype if x.dtype in SUPPORTED_DTYPES_FLOAT else torch.float16
        # weight_fp8 is [out, in] = [N, K]: consumed directly as the K-major B operand.
        w = self.weight_fp8
        if (w.dtype == torch.uint8 and x_fp8.dtype == torch.uint8 and self.in_features % 16 == 0
                and w.is_contiguous() and w.data_ptr() % 16 == 0 and x_fp8.data_ptr() % 16 == 0
                and w.device == x_fp8.device):
            # the weight prepared once: no per-call operand preparation
            w_s8, sums = self._prepared_weight()
            output = _linear_prepared(x_fp8, w_s8, sums, x_scale, self.weight_scale, self.bias, out_dtype)
        elif self.bias is None:
            output = _gemm_codes(x_fp8, self.weight_fp8, x_scale, self.weight_scale, out_dtype, _lib.B_NK)
        else:
            output = _linear_bias(x_fp8, self.weight_fp8, x_scale, self.weight_scale, self.bias, out_dtype)
        return output.view(*orig_shape[:-1], self.out_features)
