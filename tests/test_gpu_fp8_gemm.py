"""FP8 GEMM on tcgen05 against the oracle and the reference's golden outputs.

Tolerance (north star): relative Frobenius error <= 1e-2 against an fp32
reference on the same quantized operands. The int8 path accumulates exactly,
so it is also checked far tighter (<= 1e-5 in fp32 output) and bit-exactly
on integer-valued problems.
"""

import numpy as np
import pytest
import torch

from conftest import host, load_golden
from oracle import tfo_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2


def codes(M, K, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype)
    from triton_ops import quantize_fp8

    return quantize_fp8(x.cuda())


@pytest.mark.parametrize("case", sorted(load_golden("fp8_gemm")))
def test_golden_cases(cuda, case):
    from triton_ops import fp8_gemm

    c = load_golden("fp8_gemm")[case]
    qa = torch.from_numpy(c["qa"]).cuda()
    qb = torch.from_numpy(c["qb"]).cuda()
    sa = torch.tensor(float(c["sa"]), device="cuda")
    sb = torch.tensor(float(c["sb"]), device="cuda")
    out32 = host(fp8_gemm(qa, qb, sa, sb, torch.float32))
    assert O.rel_fro(out32, c["c32"]) <= 1e-5
    out16 = host(fp8_gemm(qa, qb, sa, sb))
    assert O.rel_fro(out16, np.asarray(c["c16"], np.float32)) <= 1e-3


def test_integer_exactness(cuda):
    """With sa = sb = 448/127 the output is sum_k (ua-128)(ub-128) exactly (|sum| < 2^24)."""
    from triton_ops import fp8_gemm

    rng = np.random.default_rng(1)
    for M, N, K in [(128, 256, 512), (200, 136, 1000), (7, 300, 64), (256, 512, 4096)]:
        ua = rng.integers(1, 256, (M, K), dtype=np.uint8)
        ub = rng.integers(1, 256, (K, N), dtype=np.uint8)
        s = torch.tensor(448.0 / 127.0, device="cuda")
        out = host(fp8_gemm(torch.from_numpy(ua).cuda(), torch.from_numpy(ub).cuda(), s, s, torch.float32))
        exact = (ua.astype(np.int64) - 128) @ (ub.astype(np.int64) - 128)
        assert np.abs(exact).max() < 2**24
        # alpha = fp32((448/127)^2 / fp32(448/127)^2) may differ from 1 by an ulp
        np.testing.assert_allclose(out, exact.astype(np.float64), rtol=2e-7, atol=0)


@pytest.mark.parametrize("M,N,K,splits", [(16, 2048, 33 * 128, 8),   # one cluster per tile, slices of 4 and 5 K blocks
                                          (16, 1024, 37 * 128, 9),   # partial sums + finalize, slices of 4 and 5
                                          (100, 2048, 4096, 8)])
def test_k_split_uneven_slices_exact(cuda, M, N, K, splits):
    """K split into slices that differ by one K block; none may be empty (an empty slice would add stale TMEM)."""
    from triton_ops import _lib, fp8_gemm

    assert _lib.select_tile(_lib.OP_FP8_GEMM, M, N, K, _lib.U8)[4] == splits
    rng = np.random.default_rng(M + N + K)
    ua = rng.integers(1, 256, (M, K), dtype=np.uint8)
    ub = rng.integers(1, 256, (K, N), dtype=np.uint8)
    s = torch.tensor(448.0 / 127.0, device="cuda")
    out = host(fp8_gemm(torch.from_numpy(ua).cuda(), torch.from_numpy(ub).cuda(), s, s, torch.float32))
    exact = (ua.astype(np.int64) - 128) @ (ub.astype(np.int64) - 128)
    assert np.abs(exact).max() < 2**24
    np.testing.assert_allclose(out, exact.astype(np.float64), rtol=2e-7, atol=0)
    # e4m3 operands: fp32 slice sums
    a8 = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda().to(torch.float8_e4m3fn)
    b8 = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32)).cuda().to(torch.float8_e4m3fn)
    one = torch.tensor(1.0, device="cuda")
    out8 = host(fp8_gemm(a8, b8, one, one, torch.float32))
    ref8 = a8.float().cpu().numpy().astype(np.float64) @ b8.float().cpu().numpy().astype(np.float64)
    assert O.rel_fro(out8, ref8) <= 1e-5
    assert _lib.device_error_flags() == 0


@pytest.mark.parametrize("M", [16, 128, 1024])
def test_config3_shapes(cuda, M):
    from triton_ops import fp8_gemm

    N = K = 4096
    qa, sa = codes(M, K, 10 + M)
    qb, sb = codes(K, N, 20)
    out = host(fp8_gemm(qa, qb, sa, sb, torch.float32))
    ref = O.fp8_gemm(qa.cpu().numpy(), qb.cpu().numpy(), sa.item(), sb.item(), "f32")
    assert O.rel_fro(out, ref) <= 1e-5
    out16 = host(fp8_gemm(qa, qb, sa, sb))
    assert O.rel_fro(out16, O.round_to(ref, "f16")) <= TOL


@pytest.mark.parametrize("M", [4096, 8192])
def test_config3_large_m_sampled_rows(cuda, M):
    from triton_ops import fp8_gemm

    N = K = 4096
    qa, sa = codes(M, K, 30 + M)
    qb, sb = codes(K, N, 20)
    out = fp8_gemm(qa, qb, sa, sb, torch.float32)
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(M))[:64]
    ref = O.fp8_gemm(qa[rows.cuda()].cpu().numpy(), qb.cpu().numpy(), sa.item(), sb.item(), "f32")
    assert O.rel_fro(host(out[rows.cuda()]), ref) <= 1e-5


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (33, 47, 129), (130, 260, 48), (257, 129, 272),
                                   (64, 1000, 2048), (500, 64, 100)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_ragged_shapes(cuda, M, N, K, out_dtype):
    from triton_ops import fp8_gemm

    qa, sa = codes(M, K, M + 1)
    qb, sb = codes(K, N, N + 2)
    out = fp8_gemm(qa, qb, sa, sb, out_dtype)
    assert out.dtype == out_dtype and out.shape == (M, N)
    ref = O.fp8_gemm(qa.cpu().numpy(), qb.cpu().numpy(), sa.item(), sb.item(), "f32")
    assert O.rel_fro(host(out), ref) <= (1e-5 if out_dtype == torch.float32 else TOL)


def test_float_inputs_quantize_like_reference(cuda):
    from triton_ops import fp8_gemm, quantize_fp8

    a = torch.randn(96, 320, device="cuda", dtype=torch.float16) * 0.1
    b = torch.randn(320, 160, device="cuda", dtype=torch.float16) * 0.1
    qa, sa = quantize_fp8(a)
    qb, sb = quantize_fp8(b)
    assert torch.equal(fp8_gemm(a, b), fp8_gemm(qa, qb, sa, sb))


def test_e4m3_operands(cuda):
    from triton_ops import fp8_gemm, quantize_fp8

    for M, N, K in [(128, 256, 512), (77, 130, 96), (1024, 4096, 4096)]:
        a = torch.randn(M, K, device="cuda", dtype=torch.float16)
        b = torch.randn(K, N, device="cuda", dtype=torch.float16)
        qa, sa = quantize_fp8(a, dtype=torch.float8_e4m3fn)
        qb, sb = quantize_fp8(b, dtype=torch.float8_e4m3fn)
        out = host(fp8_gemm(qa, qb, sa, sb, torch.float32))
        ref = O.fp8_gemm_e4m3(qa.view(torch.uint8).cpu().numpy(), qb.view(torch.uint8).cpu().numpy(),
                              sa.item(), sb.item(), "f32")
        assert O.rel_fro(out, ref) <= 1e-5
        # and against unquantized fp32 the e4m3 error stays at the format's level
        assert O.rel_fro(out, host(a.float() @ b.float())) <= 0.08


def test_fp8linear_matches_explicit_gemm(cuda):
    from triton_ops import FP8Linear, fp8_gemm, quantize_fp8

    torch.manual_seed(0)
    lin = FP8Linear(256, 512, bias=True).cuda()
    x = torch.randn(2, 16, 256, device="cuda", dtype=torch.float16)
    y = lin(x)
    assert y.shape == (2, 16, 512)
    qx, sx = quantize_fp8(x.view(-1, 256))
    ref = fp8_gemm(qx, lin.weight_fp8.t().contiguous(), sx, lin.weight_scale) + lin.bias
    assert torch.equal(y.view(-1, 512), ref)
    assert lin.weight_fp8.shape == (512, 256) and lin.weight_fp8.dtype == torch.uint8


def test_reference_accuracy_vs_fp16(cuda):
    """The reference's accuracy property (mean relative error vs an fp16 matmul).

    The error comes from the reference's linear 8-bit code, not from the GEMM:
    the kernel's result equals the oracle on the same codes to 1e-5, so its
    error against fp16 must equal the oracle's. (The reference's 5% bar is not
    met by the codec itself: measured 5-11% at these shapes, dominated by
    near-zero outputs.)
    """
    from triton_ops import fp8_gemm, quantize_fp8

    for M, N, K in [(64, 64, 64), (300, 200, 500), (512, 512, 512)]:
        a = torch.randn(M, K, device="cuda", dtype=torch.float16) * 0.02
        b = torch.randn(K, N, device="cuda", dtype=torch.float16) * 0.02
        ref = torch.matmul(a, b).float()
        out = fp8_gemm(a, b).float()
        err = ((out - ref).abs() / (ref.abs() + 1e-6)).mean().item()
        qa, sa = quantize_fp8(a)
        qb, sb = quantize_fp8(b)
        oracle = torch.from_numpy(O.fp8_gemm(qa.cpu().numpy(), qb.cpu().numpy(), sa.item(), sb.item(), "f16")).cuda()
        err_oracle = ((oracle - ref).abs() / (ref.abs() + 1e-6)).mean().item()
        assert abs(err - err_oracle) < 2e-3, (err, err_oracle)


def test_validation(cuda):
    from triton_ops import fp8_gemm
    from triton_ops.exceptions import ShapeMismatchError, UnsupportedDtypeError

    a = torch.zeros(8, 16, dtype=torch.uint8, device="cuda")
    s = torch.tensor(1.0, device="cuda")
    with pytest.raises(ShapeMismatchError):
        fp8_gemm(a, torch.zeros(8, 8, dtype=torch.uint8, device="cuda"), s, s)
    with pytest.raises(UnsupportedDtypeError):
        fp8_gemm(a, torch.zeros(16, 8, dtype=torch.uint8, device="cuda"), s, s, torch.int32)
    with pytest.raises(UnsupportedDtypeError):
        fp8_gemm(a, torch.zeros(16, 8, dtype=torch.float8_e4m3fn, device="cuda"), s, s)


# Shapes whose 128 x 256 tiles fill the GPU use two-CTA 256 x 256 tiles; ragged
# M leaves the second CTA's rows partly or wholly outside the matrix.
@pytest.mark.parametrize("M,N,K", [(300, 12800, 256), (1000, 4864, 384), (129, 37888, 128), (4095, 4096, 200),
                                   (256, 4096, 1024), (200, 1024, 2048), (1024, 4096, 4096),
                                   (300, 144, 208), (2000, 1040, 4112)])
def test_pair_tiles_ragged(cuda, M, N, K):
    from triton_ops import fp8_gemm

    qa, sa = codes(M, K, M + 3)
    qb, sb = codes(K, N, N + 4)
    out = fp8_gemm(qa, qb, sa, sb, torch.float32)
    rows = torch.cat([torch.arange(0, min(M, 40)), torch.arange(max(0, M - 40), M)]).unique()
    ref = O.fp8_gemm(qa[rows.cuda()].cpu().numpy(), qb.cpu().numpy(), sa.item(), sb.item(), "f32")
    assert O.rel_fro(host(out[rows.cuda()]), ref) <= 1e-5


def test_pair_tiles_e4m3_and_nk_layout(cuda):
    from triton_ops import FP8Linear, fp8_gemm, quantize_fp8

    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(520, 512, device="cuda", generator=g).half()
    b = torch.randn(512, 9472, device="cuda", generator=g).half()
    qa, sa = quantize_fp8(a, dtype=torch.float8_e4m3fn)
    qb, sb = quantize_fp8(b, dtype=torch.float8_e4m3fn)
    out = host(fp8_gemm(qa, qb, sa, sb, torch.float32))
    ref = (qa.float() / sa) @ (qb.float() / sb)
    assert O.rel_fro(out, host(ref)) <= 1e-5
    lin = FP8Linear(512, 9472).cuda()
    x = torch.randn(600, 512, device="cuda", generator=g)
    y = host(lin(x))
    xq, xs = quantize_fp8(x)
    ref = O.fp8_gemm(xq.cpu().numpy(), lin.weight_fp8.cpu().numpy().T.copy(), xs.item(), lin.weight_scale.item(), "f32")
    assert O.rel_fro(y, ref) <= 1e-5


def test_pair_and_single_cta_tiles_agree(cuda, tmp_path):
    """The same problem with two-CTA tiles switched off (TFO_B200_PAIR_MMA=0) gives identical bytes."""
    import os
    import subprocess
    import sys

    from conftest import PKG, ROOT
    from triton_ops import fp8_gemm

    qa, sa = codes(1000, 384, 11)
    qb, sb = codes(384, 4864, 12)
    np.save(tmp_path / "qa.npy", qa.cpu().numpy())
    np.save(tmp_path / "qb.npy", qb.cpu().numpy())
    prog = (
        "import sys, numpy as np, torch; sys.path[:0] = [%r, %r]\n"
        "from triton_ops import fp8_gemm\n"
        "qa = torch.from_numpy(np.load(%r)).cuda(); qb = torch.from_numpy(np.load(%r)).cuda()\n"
        "o = fp8_gemm(qa, qb, torch.tensor(%r, device='cuda'), torch.tensor(%r, device='cuda'), torch.float16)\n"
        "np.save(%r, o.cpu().numpy())\n"
    ) % (str(PKG), str(ROOT), str(tmp_path / "qa.npy"), str(tmp_path / "qb.npy"), sa.item(), sb.item(),
         str(tmp_path / "single.npy"))
    env = dict(os.environ, TFO_B200_PAIR_MMA="0")
    subprocess.run([sys.executable, "-c", prog], check=True, env=env, timeout=300)
    single = np.load(tmp_path / "single.npy")
    pair = fp8_gemm(qa, qb, sa, sb, torch.float16).cpu().numpy()
    np.testing.assert_array_equal(pair.view(np.uint16), single.view(np.uint16))


@pytest.mark.parametrize("M", [16, 256, 1000])
@pytest.mark.parametrize("xdt,bdt", [(torch.float16, torch.float32), (torch.bfloat16, torch.float32),
                                     (torch.float32, torch.float32), (torch.float16, torch.float16)])
def test_fp8linear_bias_in_epilogue(cuda, M, xdt, bdt):
    """FP8Linear's bias, added in the GEMM epilogue, equals fp8_gemm(...) + bias bit for bit (dtype promotion too)."""
    from triton_ops import FP8Linear
    from triton_ops import _lib
    from triton_ops.kernels.fp8_gemm import _gemm_codes
    from triton_ops.kernels.fp8_quantize import quantize_fp8

    g = torch.Generator(device="cuda").manual_seed(M)
    lin = FP8Linear(512, 4096, bias=True).cuda()
    with torch.no_grad():
        lin.bias.copy_(torch.randn(4096, device="cuda", generator=g))
    lin.bias.data = lin.bias.data.to(bdt)
    x = torch.randn(M, 512, device="cuda", generator=g).to(xdt)
    y = lin(x)
    xq, xs = quantize_fp8(x)
    ref = _gemm_codes(xq, lin.weight_fp8, xs, lin.weight_scale, xdt, _lib.B_NK) + lin.bias
    assert y.dtype == ref.dtype and y.shape == ref.shape
    assert torch.equal(y, ref)


@pytest.mark.parametrize("M", [1, 16, 300, 2048])
@pytest.mark.parametrize("with_bias", [False, True])
def test_prepared_weight_linear_equals_linear(cuda, M, with_bias):
    """tfo_fp8_linear_prepared (weight sign-flipped and summed once) gives tfo_fp8_linear's bits, for M on
    both sides of N (where tfo_fp8_linear prepares A, and where it prepares the weight per call)."""
    from triton_ops import _lib, quantize_fp8
    from triton_ops.kernels.fp8_gemm import _linear_bias, _gemm_codes, _linear_prepared

    N, K = 1024, 512
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = 0.05 * torch.randn(N, K, device="cuda", generator=g)
    qx, sx = quantize_fp8(x)
    qw, sw = quantize_fp8(w)
    w_s8 = torch.empty(N, K, dtype=torch.int8, device="cuda")
    sums = torch.empty(N, dtype=torch.int32, device="cuda")
    _lib.call("tfo_fp8_prepare_weight", qw.data_ptr(), N, K, w_s8.data_ptr(), sums.data_ptr(), _lib.stream_of(qw))
    ref_s8 = (qw.cpu().numpy().astype(np.int32) - 128).astype(np.int8)
    np.testing.assert_array_equal(w_s8.cpu().numpy(), ref_s8)
    np.testing.assert_array_equal(sums.cpu().numpy(), ref_s8.astype(np.int64).sum(axis=1))
    bias = (0.1 * torch.randn(N, device="cuda", generator=g)).float() if with_bias else None
    got = _linear_prepared(qx, w_s8, sums, sx, sw, bias, torch.float16)
    want = (_linear_bias(qx, qw, sx, sw, bias, torch.float16) if with_bias
            else _gemm_codes(qx, qw, sx, sw, torch.float16, _lib.B_NK))
    assert got.dtype == want.dtype and torch.equal(got, want)
    assert _lib.device_error_flags() == 0


def test_fp8linear_prepared_and_unaligned_in_features(cuda):
    """FP8Linear uses the prepared weight when in_features % 16 == 0 (equal to the explicit GEMM), the
    per-call path otherwise; modifying weight_fp8 in place refreshes the prepared copy."""
    from triton_ops import FP8Linear, fp8_gemm, quantize_fp8

    torch.manual_seed(1)
    for K in (256, 100):
        lin = FP8Linear(K, 384, bias=True).cuda()
        x = torch.randn(3, 7, K, device="cuda", dtype=torch.float16)
        y = lin(x)
        qx, sx = quantize_fp8(x.view(-1, K))
        ref = fp8_gemm(qx, lin.weight_fp8.t().contiguous(), sx, lin.weight_scale) + lin.bias
        assert torch.equal(y.view(-1, 384), ref)
    lin2 = FP8Linear(256, 384, bias=False).cuda()
    x2 = torch.randn(5, 256, device="cuda", dtype=torch.float16)
    y1 = lin2(x2)
    lin2.weight_fp8.fill_(128)  # in place (code 128 decodes to 0): the next forward must see it
    assert torch.equal(lin2(x2), torch.zeros_like(y1))


# Few-row products with a K-major [N, K] B (FP8Linear's layout) against the
# oracle: codec (exact int32 sums) and e4m3, ragged N and M = 1.
@pytest.mark.parametrize("M,N,K", [(16, 4096, 4096), (1, 4096, 1024), (32, 2390, 4096), (7, 3000, 272)])
@pytest.mark.parametrize("qdt", [torch.uint8, torch.float8_e4m3fn])
def test_few_rows_nk_b_match_oracle(cuda, M, N, K, qdt):
    from triton_ops import _lib, quantize_fp8
    from triton_ops.kernels.fp8_gemm import _gemm_codes

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    qa, sa = quantize_fp8(torch.randn(M, K, device="cuda", generator=g).half(), dtype=qdt)
    qb, sb = quantize_fp8(torch.randn(N, K, device="cuda", generator=g).half(), dtype=qdt)  # [N, K]
    out = host(_gemm_codes(qa, qb, sa, sb, torch.float32, _lib.B_NK))
    a_u8, b_u8 = qa.view(torch.uint8).cpu().numpy(), qb.view(torch.uint8).cpu().numpy()
    if qdt == torch.uint8:
        ref = O.fp8_gemm(a_u8, b_u8.T, sa.item(), sb.item(), "f32")
    else:
        ref = O.fp8_gemm_e4m3(a_u8, b_u8.T, sa.item(), sb.item(), "f32")
    assert O.rel_fro(out, ref) <= 1e-5
    out16 = host(_gemm_codes(qa, qb, sa, sb, torch.float16, _lib.B_NK))
    assert O.rel_fro(out16, ref) <= 1e-3
    assert _lib.device_error_flags() == 0


@pytest.mark.parametrize("M", [1, 16, 32])
def test_prepared_linear_with_bias_matches_oracle(cuda, M):
    """FP8Linear(4096, 4096, bias) at decode sizes (prepared int8 weight, raw u8 activations,
    per-column correction, bias in the epilogue) against the oracle's GEMM plus the bias."""
    from triton_ops import FP8Linear, quantize_fp8

    torch.manual_seed(M)
    lin = FP8Linear(4096, 4096, bias=True).cuda()
    with torch.no_grad():
        lin.bias.normal_()
    x = torch.randn(M, 4096, device="cuda", dtype=torch.float16)
    y = lin(x)
    y = lin(x)  # second call: the prepared weight (the first call quantizes and prepares it)
    qx, sx = quantize_fp8(x)
    ref = O.fp8_gemm(qx.cpu().numpy(), lin.weight_fp8.cpu().numpy().T, sx.item(), lin.weight_scale.item(), "f16")
    ref = O.round_to(ref + host(lin.bias), "f32")  # fp16 product + fp32 bias -> fp32 (torch's promotion)
    assert y.dtype == torch.float32 and y.shape == (M, 4096)
    assert O.rel_fro(host(y), ref) <= 1e-3
