"""Per-token / per-channel FP8 scales: scale vectors applied in the GEMM epilogue.

The reference's FP8Format.compute_scale_per_channel (models.py:301-314) is a
torch expression; its quantize/dequantize kernels read one scale. Here the
per-channel scale runs natively, quantize/dequantize accept one scale per
row, and fp8_gemm applies per-row A and per-column B scale vectors.
"""

import numpy as np
import pytest
import torch

from conftest import host
from oracle import tfo_oracle as O

pytestmark = pytest.mark.gpu


def torch_per_channel(t, dim):
    """The reference's expression, verbatim in meaning."""
    max_abs = t.abs().amax(dim=dim, keepdim=True)
    max_abs = torch.where(max_abs == 0, torch.ones_like(max_abs), max_abs)
    return 448.0 / max_abs


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_compute_scale_per_channel_native_equals_reference_expression(cuda, dtype):
    from triton_ops import FP8Format

    x = (torch.randn(300, 517, device="cuda") * 3).to(dtype)
    x[7] = 0  # a zero channel: scale 448
    got = FP8Format.compute_scale_per_channel(x, dim=-1)
    ref = torch_per_channel(x, -1)
    assert got.dtype == ref.dtype and got.shape == ref.shape == (300, 1)
    assert torch.equal(got, ref)
    assert torch.equal(FP8Format.compute_scale_per_channel(x, dim=0), torch_per_channel(x, 0))  # torch path


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("code", [torch.uint8, torch.float8_e4m3fn])
@pytest.mark.parametrize("shape", [(4096, 4096), (2, 3, 256), (37, 100), (5, 8)])
def test_quantize_per_token_equals_scale_then_quantize(cuda, dtype, code, shape):
    """One launch gives the bytes of compute_scale_per_channel(x, -1) followed by quantize_fp8(x, scales):
    the same [..., 1] scales in x's dtype (the reference's torch expression) and the same codes. Rows of
    whole 16-byte vectors (4096, 256 columns) and element-wise rows (100, 8 columns); a zero row gets 448, a
    row of 1e-6 an infinite fp16 scale (the clamped encode path; finite rows take the in-range one)."""
    from triton_ops import FP8Format, quantize_fp8, quantize_fp8_per_token

    torch.manual_seed(sum(shape))
    x = (torch.randn(*shape, device="cuda") * torch.rand(*shape[:-1], 1, device="cuda") * 50).to(dtype)
    x.view(-1, shape[-1])[1] = 0
    x.view(-1, shape[-1])[2] = 1e-6
    q, s = quantize_fp8_per_token(x, dtype=code)
    s_ref = FP8Format.compute_scale_per_channel(x, dim=-1)
    q_ref, _ = quantize_fp8(x, s_ref, dtype=code)
    assert s.dtype == s_ref.dtype == dtype and s.shape == s_ref.shape == (*shape[:-1], 1)
    assert torch.equal(s, s_ref) and torch.equal(s, torch_per_channel(x, -1))
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    if code == torch.uint8:
        np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(host(x), host(s)))


def test_quantize_per_token_one_launch(cuda):
    """[4096, 4096] fp16: one kernel launch (the two-call form takes three)."""
    from triton_ops import _lib, quantize_fp8_per_token

    x = torch.randn(4096, 4096, device="cuda").half()
    quantize_fp8_per_token(x)
    torch.cuda.synchronize()
    n0 = _lib.kernel_launches()
    quantize_fp8_per_token(x)
    assert _lib.kernel_launches() - n0 == 1
    assert _lib.device_error_flags() == 0


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
def test_quantize_dequantize_per_row(cuda, dt):
    from triton_ops import FP8Format, dequantize_fp8, quantize_fp8

    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    x = (torch.randn(257, 300, device="cuda") * torch.linspace(0.01, 100, 257, device="cuda")[:, None]).to(tdt)
    s = FP8Format.compute_scale_per_channel(x.float(), dim=-1)  # fp32 [257, 1]
    q, s_back = quantize_fp8(x, s)
    assert s_back is s
    xn, sn = host(x), host(s)
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(xn, sn))
    for od, name in ((torch.float16, "f16"), (torch.float32, "f32"), (torch.bfloat16, "bf16")):
        np.testing.assert_array_equal(host(dequantize_fp8(q, s, od)), O.dequantize_ref(q.cpu().numpy(), sn, name))
    q8, _ = quantize_fp8(x, s, dtype=torch.float8_e4m3fn)
    ref8 = (x.float() * s).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(q8.view(torch.uint8), ref8.view(torch.uint8))
    d8 = dequantize_fp8(q8, s, torch.float32)
    assert torch.equal(d8, ref8.float() / s)


@pytest.mark.parametrize("M", [16, 256, 1000, 4096])
@pytest.mark.parametrize("code", [torch.uint8, torch.float8_e4m3fn])
def test_gemm_with_token_and_channel_scales(cuda, M, code):
    from triton_ops import FP8Format, fp8_gemm, quantize_fp8

    g = torch.Generator(device="cuda").manual_seed(M)
    K, N = 1024, 2048
    a = torch.randn(M, K, device="cuda", generator=g) * torch.linspace(0.1, 10, M, device="cuda")[:, None]
    b = torch.randn(K, N, device="cuda", generator=g) * torch.linspace(0.1, 10, N, device="cuda")[None, :]
    sa = FP8Format.compute_scale_per_channel(a, dim=-1)            # [M, 1] per token
    sb = FP8Format.compute_scale_per_channel(b.t().contiguous(), dim=-1).reshape(1, N)  # per output channel
    qa, _ = quantize_fp8(a, sa, dtype=code)
    qb, _ = quantize_fp8(b.t().contiguous(), sb.reshape(N, 1), dtype=code)
    qb = qb.t().contiguous()  # [K, N] codes of B
    out = host(fp8_gemm(qa, qb, sa, sb, torch.float32))

    def dec(q):
        if q.dtype == torch.uint8:
            return (q.cpu().numpy().astype(np.float64) - 128) / 127 * 448
        return q.float().cpu().numpy().astype(np.float64)

    ref = (dec(qa) / host(sa).astype(np.float64)) @ (dec(qb) / host(sb).astype(np.float64))
    assert O.rel_fro(out, ref) <= 1e-5
    # one-sided: per-token A scales with a per-tensor B scale
    sb1 = torch.tensor(float(sb.min().item()), device="cuda")
    qb1, _ = quantize_fp8(b, sb1, dtype=code)
    out1 = host(fp8_gemm(qa, qb1, sa, sb1, torch.float32))
    ref1 = (dec(qa) / host(sa).astype(np.float64)) @ (dec(qb1) / float(sb1.item()))
    assert O.rel_fro(out1, ref1) <= 1e-5


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("rows,cols", [(1, 16), (3, 48), (37, 1040), (16, 4096), (3, 8208)])
def test_per_row_vector_and_scalar_paths(cuda, dt, rows, cols):
    """Rows of whole 16-element chunks on 16-byte boundaries take the vectorised per-row kernels;
    the same values one element off a 16-byte boundary take the element-wise ones. Both equal the
    oracle (codes, decoded values) and torch's expression (scales), NaN/inf elements and a zero
    row included."""
    from triton_ops import FP8Format, dequantize_fp8, quantize_fp8

    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    g = torch.Generator().manual_seed(rows * cols)
    x = (torch.randn(rows, cols, generator=g) * torch.logspace(-2, 2, rows)[:, None]).to(tdt).cuda()
    if rows > 2:
        x[rows // 2] = 0
    s = FP8Format.compute_scale_per_channel(x, dim=-1)
    assert torch.equal(s, torch_per_channel(x, -1))
    s32 = s.float()
    xs = x.clone()
    xs[0, 1] = float("inf")
    xs[0, cols - 1] = float("nan")
    flat = torch.empty(rows * cols + 8, dtype=tdt, device="cuda")
    off = flat[1:1 + rows * cols].view(rows, cols)  # 2 or 4 bytes past a 16-byte boundary
    off.copy_(xs)
    xn, sn = host(xs), host(s32)
    for src in (xs, off):
        q, _ = quantize_fp8(src, s32)
        np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(xn, sn))
        for od, name in ((torch.float16, "f16"), (torch.float32, "f32"), (torch.bfloat16, "bf16")):
            np.testing.assert_array_equal(host(dequantize_fp8(q, s32, od)), O.dequantize_ref(q.cpu().numpy(), sn, name))
        q8, _ = quantize_fp8(src, s32, dtype=torch.float8_e4m3fn)
        ref8 = (xs.float() * s32).clamp(-448, 448).to(torch.float8_e4m3fn)
        assert torch.equal(q8.view(torch.uint8), ref8.view(torch.uint8))
        d8 = dequantize_fp8(q8, s32, torch.float32)
        torch.testing.assert_close(d8, ref8.float() / s32, rtol=0, atol=0, equal_nan=True)
    qo = torch.empty(rows * cols + 16, dtype=torch.uint8, device="cuda")[3:3 + rows * cols].view(rows, cols)
    q, _ = quantize_fp8(xs, s32)
    qo.copy_(q)
    np.testing.assert_array_equal(host(dequantize_fp8(qo, s32, torch.float32)),
                                  O.dequantize_ref(q.cpu().numpy(), sn, "f32"))
