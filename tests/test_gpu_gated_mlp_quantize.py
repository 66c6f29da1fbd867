"""Gated MLP -> 8-bit codes: bytes equal to quantize_fp8(fused_gated_mlp(...)).

No counterpart in the reference; the contract is exact equality with the
reference's two ops in sequence, on every path: codes written by the MLP
epilogue (given scale), rows + epilogue maxima feeding the encode (dynamic
scale), and the CUDA-core layouts (the two ops).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def mlp_inputs(M, N, K, xd, wd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(1, M, K, device="cuda", generator=g).to(DT[xd])
    wg = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(DT[wd])
    wu = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(DT[wd])
    return x, wg, wu


def check(M, N, K, xd="f16", wd="f16", act="silu", scale=None, dtype=torch.uint8, seed=0, launches=None):
    from triton_ops import _lib, fused_gated_mlp, fused_gated_mlp_quantize, quantize_fp8

    x, wg, wu = mlp_inputs(M, N, K, xd, wd, seed)
    st = None if scale is None else torch.tensor(scale, device="cuda")
    n0 = _lib.kernel_launches()
    q, s = fused_gated_mlp_quantize(x, wg, wu, act, st, dtype=dtype)
    n1 = _lib.kernel_launches()
    q_ref, s_ref = quantize_fp8(fused_gated_mlp(x, wg, wu, act), st, dtype=dtype)
    assert q.dtype == dtype and q.shape == (1, M, N)
    assert s.item() == s_ref.item()
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    if launches is not None:
        assert n1 - n0 == launches, n1 - n0
    assert _lib.device_error_flags() == 0


@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
def test_codes_from_the_epilogue_given_scale(cuda, act):
    check(2048, 11264, 4096, act=act, scale=40.0, seed=1, launches=1)


def test_dynamic_scale_from_epilogue_maxima(cuda):
    check(2048, 11264, 4096, seed=2, launches=2)
    check(300, 1000, 640, xd="bf16", wd="bf16", seed=3, launches=2)
    check(100, 200, 136, seed=4, launches=2)  # one-CTA tiles


def test_e4m3_and_fp32_weights(cuda):
    check(1000, 2048, 1024, scale=0.5, dtype=torch.float8_e4m3fn, seed=5, launches=1)
    check(1000, 2048, 1024, dtype=torch.float8_e4m3fn, seed=6, launches=2)
    check(200, 96, 256, xd="f16", wd="f32", seed=7)  # tf32 path (fp32 copies of x first)


def test_cuda_core_layout_and_empty(cuda):
    from triton_ops import fused_gated_mlp_quantize

    check(33, 65, 100, seed=8)  # K % 8 != 0: CUDA-core MLP, then the quantize
    check(33, 65, 100, scale=3.0, seed=9)
    x = torch.empty(1, 0, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 64, device="cuda", dtype=torch.float16)
    q, s = fused_gated_mlp_quantize(x, w, w)
    assert q.shape == (1, 0, 32) and s.item() == 1.0
