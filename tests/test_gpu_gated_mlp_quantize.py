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


# --- against the oracle chain -------------------------------------------------
# Reference chain served by the fused op: gated_mlp_reference (gated_mlp.py:221-251)
# then the quantize oracle (fp8_quantize.py:258-287, scale rule models.py:282-299).
_ORACLE_CACHE = {}


def config4_oracle(act):
    """Config 4 inputs (x [2, 1024, 4096] fp16 N(0, 1), W [11264, 4096] fp16 N(0, 0.02))
    and the oracle's fp16 output for all 2048 rows (float64 sums)."""
    import numpy as np

    from conftest import host
    from oracle import tfo_oracle as O

    g = torch.Generator(device="cuda").manual_seed(41)
    x = torch.randn(2, 1024, 4096, device="cuda", generator=g).half()
    wg = (0.02 * torch.randn(11264, 4096, device="cuda", generator=g)).half()
    wu = (0.02 * torch.randn(11264, 4096, device="cuda", generator=g)).half()
    if act not in _ORACLE_CACHE:  # 92 MB per activation, computed once per session
        _ORACLE_CACHE[act] = O.gated_mlp(host(x).reshape(-1, 4096), host(wg), host(wu), act, "f16")
    return x, wg, wu, np.asarray(_ORACLE_CACHE[act], np.float32)


def assert_codes_follow_oracle(got_codes, gpu_out, ref_out, scale):
    """Codes equal quantize_ref(oracle output, scale); where they differ, the kernel's
    fp16 output differs from the oracle's (fp32 vs float64 sums) and by one code step."""
    import numpy as np

    from oracle import tfo_oracle as O

    ref_codes = O.quantize_ref(ref_out, np.float32(scale))
    diff = got_codes.astype(np.int32) - ref_codes.astype(np.int32)
    assert np.abs(diff).max() <= 1
    off = diff != 0
    assert np.mean(off) < 1e-3, np.mean(off)
    assert np.all(gpu_out[off] != ref_out[off])  # every code difference comes from an fp16 rounding difference


@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
def test_dynamic_scale_matches_oracle_config4(cuda, act):
    import numpy as np

    from conftest import host
    from oracle import tfo_oracle as O
    from triton_ops import fused_gated_mlp, fused_gated_mlp_quantize

    x, wg, wu, ref = config4_oracle(act)
    q, s = fused_gated_mlp_quantize(x, wg, wu, act)
    out = host(fused_gated_mlp(x, wg, wu, act)).reshape(-1, 11264)
    s_ref = O.compute_scale(ref)
    # amax is taken over fp16 outputs: the kernel's and the oracle's maxima agree
    # to within one fp16 ulp, so the scales agree to within 2^-10 relative
    assert abs(float(s.item()) / float(s_ref) - 1.0) <= 2.0**-10
    assert float(s.item()) == float(O.compute_scale(out))
    assert_codes_follow_oracle(q.cpu().numpy().reshape(-1, 11264), out, ref, s.item())


@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
def test_given_scale_matches_oracle_config4_sampled_rows(cuda, act):
    from conftest import host
    from triton_ops import fused_gated_mlp, fused_gated_mlp_quantize

    x, wg, wu, ref = config4_oracle(act)
    sc = 40.0
    q, s = fused_gated_mlp_quantize(x, wg, wu, act, torch.tensor(sc, device="cuda"))
    assert s.item() == sc
    rows = torch.randperm(2048, generator=torch.Generator().manual_seed(3))[:256]
    out = host(fused_gated_mlp(x, wg, wu, act)).reshape(-1, 11264)[rows.numpy()]
    got = q.reshape(-1, 11264)[rows.cuda()].cpu().numpy()
    assert_codes_follow_oracle(got, out, ref[rows.numpy()], sc)
