"""Fused gated MLP: ``gate_proj(x) * act(up_proj(x))``.

``fused_gated_mlp`` launches the tcgen05 kernel behind ``tfo_gated_mlp``
(csrc/gated_mlp.cu): the gate and up projections share each x tile, both
accumulate in TMEM in fp32, and the epilogue applies the activation to the
UP projection and multiplies by the gate, as the reference does
(triton_ops/kernels/gated_mlp.py:128-134, 243-249). Activations: "silu",
"gelu" (erf form, the reference's) and "gelu_tanh" (extension).

``gated_mlp_reference`` restates the reference's PyTorch oracle (:221-251)
for tests; the op never calls it.
"""

from __future__ import annotations

import torch

from triton_ops import _lib
from triton_ops.kernels._native import NativeKernel
from triton_ops.validation import validate_gated_mlp_inputs

fused_gated_mlp_kernel = NativeKernel(
    "fused_gated_mlp_kernel", "tfo_gated_mlp", "shared A tile, two TMEM accumulators, activation in the epilogue"
)
fused_gated_mlp_quantize_kernel = NativeKernel(
    "fused_gated_mlp_quantize_kernel", "tfo_gated_mlp_quantize", "gated MLP with 8-bit codes from the epilogue"
)


def fused_gated_mlp(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    activation: str = "silu",
) -> torch.Tensor:
    """Gated MLP over x [batch, seq_len, hidden] with weights [intermediate, hidden].

    Returns [batch, seq_len, intermediate] in x's dtype.
    """
    batch_size, seq_len, hidden_dim, intermediate_dim = validate_gated_mlp_inputs(x, gate_weight, up_weight, activation)
    out = torch.empty(batch_size, seq_len, intermediate_dim, dtype=x.dtype, device=x.device)
    M = batch_size * seq_len
    if out.numel() == 0:
        return out
    x_code = _lib.dtype_code(x.dtype, "x")
    w_code = _lib.dtype_code(gate_weight.dtype, "gate_weight")
    if up_weight.dtype != gate_weight.dtype:
        up_weight = up_weight.to(gate_weight.dtype)
    lib = _lib.load()
    ws_bytes = lib.tfo_gated_mlp_workspace_bytes(M, intermediate_dim, hidden_dim, x_code, w_code)
    ws = _lib.workspace(ws_bytes, x.device)
    _lib.call(
        "tfo_gated_mlp", x.data_ptr(), gate_weight.data_ptr(), up_weight.data_ptr(), out.data_ptr(), M,
        intermediate_dim, hidden_dim, x_code, w_code, _lib.ACT_CODE[activation], ws.data_ptr(), ws.numel(),
        _lib.stream_of(x),
    )
    return out


def fused_gated_mlp_quantize(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    activation: str = "silu",
    scale: torch.Tensor = None,
    *,
    dtype: torch.dtype = torch.uint8,
) -> tuple:
    """Gated MLP whose output comes back as 8-bit codes, for an FP8 down-projection.

    Returns ``(codes, scale)`` equal, byte for byte, to
    ``quantize_fp8(fused_gated_mlp(x, gate_weight, up_weight, activation), scale, dtype=dtype)``.
    With a given `scale` the MLP epilogue writes the codes directly (the
    [M, intermediate] output never reaches memory); with ``scale=None`` the
    epilogue also records per-warp maxima of the output, from which the encode
    pass derives the scale without a separate amax read. The reference has no
    such op; its roadmap chains the gated MLP into an ``FP8Linear``.
    """
    from triton_ops.exceptions import UnsupportedDtypeError
    from triton_ops.kernels.fp8_quantize import _CODE_DTYPES, _scale_f32

    batch_size, seq_len, hidden_dim, intermediate_dim = validate_gated_mlp_inputs(x, gate_weight, up_weight, activation)
    if dtype not in _CODE_DTYPES:
        raise UnsupportedDtypeError(f"codes dtype must be one of {_CODE_DTYPES}, got {dtype}", dtype=dtype,
                                    supported_dtypes=list(_CODE_DTYPES))
    dev = x.device
    if up_weight.dtype != gate_weight.dtype:
        up_weight = up_weight.to(gate_weight.dtype)
    codes = torch.empty(batch_size, seq_len, intermediate_dim, dtype=dtype, device=dev)
    s32 = scale_out = None
    if scale is None:
        scale = scale_out = torch.empty((), dtype=torch.float32, device=dev)
    else:
        s32 = _scale_f32(scale.to(dev))
    M = batch_size * seq_len
    x_code = _lib.dtype_code(x.dtype, "x")
    w_code = _lib.dtype_code(gate_weight.dtype, "gate_weight")
    lib = _lib.load()
    ws_bytes = lib.tfo_gated_mlp_quantize_workspace_bytes(x.data_ptr(), gate_weight.data_ptr(), up_weight.data_ptr(), M,
                                                          intermediate_dim, hidden_dim, x_code, w_code,
                                                          int(s32 is not None))
    ws = _lib.workspace(ws_bytes, dev)
    _lib.call(
        "tfo_gated_mlp_quantize", x.data_ptr(), gate_weight.data_ptr(), up_weight.data_ptr(), codes.data_ptr(), M,
        intermediate_dim, hidden_dim, x_code, w_code, _lib.ACT_CODE[activation], _lib.ptr(s32), _lib.ptr(scale_out),
        _lib.dtype_code(dtype), ws.data_ptr(), ws.numel(), _lib.stream_of(x),
    )
    return codes, scale


def gated_mlp_reference(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    activation: str = "silu",
) -> torch.Tensor:
    """PyTorch restatement of the reference oracle (fp32 projections, activation on up)."""
    gate = torch.nn.functional.linear(x.float(), gate_weight.float())
    up = torch.nn.functional.linear(x.float(), up_weight.float())
    if activation == "silu":
        act = torch.nn.functional.silu(up)
    elif activation == "gelu_tanh":
        act = torch.nn.functional.gelu(up, approximate="tanh")
    else:
        act = torch.nn.functional.gelu(up)
    return (gate * act).to(x.dtype)


class FusedGatedMLP(torch.nn.Module):
    """Module form: fp32 gate/up weights [intermediate, hidden], N(0, 0.02) init."""

    def __init__(self, hidden_dim: int, intermediate_dim: int, activation: str = "silu"):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.activation = activation
        self.gate_weight = torch.nn.Parameter(torch.randn(intermediate_dim, hidden_dim) * 0.02)
        self.up_weight = torch.nn.Parameter(torch.randn(intermediate_dim, hidden_dim) * 0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_gated_mlp(x, self.gate_weight, self.up_weight, self.activation)
