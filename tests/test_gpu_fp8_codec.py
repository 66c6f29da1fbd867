"""FP8 codec on the GPU: bit-exact against the oracle and the reference's golden outputs."""

import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, NAME_DT, dev_tensor, host, load_golden
from oracle import tfo_oracle as O

pytestmark = pytest.mark.gpu


def f32bits(v):
    return int(np.float32(v).view(np.uint32))


@pytest.mark.parametrize("case", sorted(load_golden("fp8_codec")))
def test_golden_cases_bit_exact(cuda, case):
    from triton_ops import dequantize_fp8, quantize_fp8

    c = load_golden("fp8_codec")[case]
    xd = NAME_DT[str(c["x_dtype"])]
    x = dev_tensor(c["x"], xd)
    given = float(c["given_scale"])
    scale_in = None if np.isnan(given) else torch.tensor(given, device="cuda")
    q, s = quantize_fp8(x, scale_in)
    assert q.dtype == torch.uint8 and q.shape == x.shape
    assert f32bits(s.item()) == f32bits(c["scale"])
    np.testing.assert_array_equal(q.cpu().numpy(), c["q"])
    dq16 = dequantize_fp8(q, s, torch.float16)
    dq32 = dequantize_fp8(q, s, torch.float32)
    np.testing.assert_array_equal(host(dq16), np.asarray(c["dq_f16"], np.float32))
    np.testing.assert_array_equal(host(dq32), c["dq_f32"])
    dqb = dequantize_fp8(q, s, torch.bfloat16)
    np.testing.assert_array_equal(host(dqb), O.dequantize_ref(c["q"], c["scale"], "bf16"))


def test_full_size_config2_digest(cuda):
    """The 4096 x 4096 N(0,1) tensor with 0.1% +-200 outliers: codes, scale and round trip."""
    from test_oracle_golden import full_codec_input
    from triton_ops import dequantize_fp8, quantize_fp8

    x_np, meta = full_codec_input()
    x = torch.from_numpy(x_np).cuda()
    q, s = quantize_fp8(x)
    assert f32bits(s.item()) == meta["scale_bits"]
    assert hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == meta["q_sha256"]
    dq = dequantize_fp8(q, s, torch.float16)
    assert hashlib.sha256(dq.cpu().numpy().tobytes()).hexdigest() == meta["dq_f16_sha256"]


def test_every_threshold_neighbourhood(cuda):
    """fp32 values within 64 ulps of every code boundary (scale 1) encode exactly as the oracle."""
    from triton_ops import quantize_fp8

    centres = np.array([(k + 0.5) * 448.0 / 127.0 for k in range(-128, 128)], dtype=np.float32)
    offs = np.arange(-64, 65, dtype=np.int32)
    bits = centres.view(np.int32)[:, None] + offs[None, :]
    vals = bits.astype(np.int32).view(np.float32).ravel()
    extra = np.array([0.0, -0.0, 448.0, -448.0, 448.1, -1e38, 3e38, np.inf, -np.inf, np.nan, 1e-45, -1e-45],
                     dtype=np.float32)
    vals = np.concatenate([vals, extra])
    q, _ = quantize_fp8(torch.from_numpy(vals).cuda(), torch.tensor(1.0, device="cuda"))
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(vals, 1.0))


@pytest.mark.parametrize("scale", [1.0, 2.24, 0.001953125, 37.5, 448.0 / 65504.0])
def test_all_fp16_bit_patterns(cuda, scale):
    from triton_ops import quantize_fp8

    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    q, _ = quantize_fp8(torch.from_numpy(allh.copy()).cuda(), torch.tensor(scale, device="cuda"))
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(allh.astype(np.float32), np.float32(scale)))


def test_all_bf16_bit_patterns(cuda):
    from triton_ops import quantize_fp8

    allb = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    xb = torch.from_numpy(allb.copy()).cuda().bfloat16()
    q, _ = quantize_fp8(xb, torch.tensor(0.75, device="cuda"))
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(allb, np.float32(0.75)))


# sizes on both quantize paths: shared-memory resident (up to ~34 MB) and L2 re-read
@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, 4097, 1 << 20, (1 << 20) + 7, 3_000_001, 9_000_000])
@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_dynamic_scale_sizes(cuda, n, dtype):
    from triton_ops import FP8Format, quantize_fp8

    rng = np.random.default_rng(n)
    x = O.round_to((rng.standard_normal(n) * 7).astype(np.float32), dtype)
    xt = dev_tensor(x, dtype)
    q, s = quantize_fp8(xt)
    s_ref = O.compute_scale(x)
    assert f32bits(s.item()) == f32bits(s_ref)
    assert f32bits(FP8Format.compute_scale(xt).item()) == f32bits(s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))


def test_unaligned_views(cuda):
    from triton_ops import dequantize_fp8, quantize_fp8

    base = torch.randn(1000, device="cuda", dtype=torch.float16)
    x = base[3:998]  # 6-byte offset: scalar path
    q, s = quantize_fp8(x)
    xn = host(x)
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(xn, O.compute_scale(xn)))
    qq = torch.cat([torch.zeros(1, dtype=torch.uint8, device="cuda"), q])[1:]
    np.testing.assert_array_equal(host(dequantize_fp8(qq, s)), O.dequantize_ref(q.cpu().numpy(), s.item(), "f16"))


def test_zero_nan_and_scale_edge_cases(cuda):
    from triton_ops import FP8Format, dequantize_fp8, quantize_fp8

    z = torch.zeros(100, device="cuda", dtype=torch.float16)
    q, s = quantize_fp8(z)
    assert s.item() == 1.0 and torch.all(q == 128)
    assert torch.equal(dequantize_fp8(q, s), z)
    xn = torch.randn(64, device="cuda")
    xn[5] = float("nan")
    s = FP8Format.compute_scale(xn)
    assert np.isnan(s.item())
    xi = torch.randn(64, device="cuda")
    xi[7] = float("inf")
    assert FP8Format.compute_scale(xi).item() == 0.0


def test_scale_given_on_other_dtype_and_shape(cuda):
    from triton_ops import quantize_fp8

    x = torch.randn(32, 32, device="cuda", dtype=torch.float16)
    q1, _ = quantize_fp8(x, torch.tensor([2.5], device="cuda", dtype=torch.float64))
    q2, _ = quantize_fp8(x, torch.tensor(2.5, device="cuda"))
    assert torch.equal(q1, q2)


def test_overflow_handling(cuda):
    from triton_ops.kernels.fp8_quantize import quantize_fp8_with_overflow_handling

    t = torch.full((100,), 1000.0, device="cuda", dtype=torch.float16)
    q, s = quantize_fp8_with_overflow_handling(t)
    assert s < 1.0
    assert torch.all(q == 255)
    # 1 -> 0.5 -> 0.25: 1000 * 0.25 = 250 <= 448 on the third check
    q2, s2 = quantize_fp8_with_overflow_handling(t, torch.tensor(1.0, device="cuda"))
    assert s2.item() == 0.25
    np.testing.assert_array_equal(q2.cpu().numpy(), O.quantize_ref(host(t), 0.25))
    # 4 -> 2 -> 1 -> 0.5: never in range after 3 halvings, as in the reference
    from triton_ops.exceptions import NumericalOverflowError

    with pytest.raises(NumericalOverflowError) as ei:
        quantize_fp8_with_overflow_handling(t, torch.tensor(4.0, device="cuda"))
    assert ei.value.attempts == 3 and ei.value.scale == 0.5


def test_reference_round_trip_property(cuda):
    """The reference's round-trip test: 95% of elements within 15% relative error."""
    from triton_ops import dequantize_fp8, quantize_fp8

    for M, N in [(16, 16), (100, 37), (512, 512)]:
        t = torch.randn(M, N, device="cuda", dtype=torch.float16) * 10.0
        q, s = quantize_fp8(t)
        d = dequantize_fp8(q, s)
        rel = (t.float() - d.float()).abs() / (t.float().abs() + 1e-6)
        assert (rel < 0.15).float().mean() > 0.8  # linear code: small values lose precision


@pytest.mark.parametrize("case", sorted(load_golden("fp8_e4m3")))
def test_e4m3_golden(cuda, case):
    from triton_ops import quantize_fp8

    c = load_golden("fp8_e4m3")[case]
    xd = NAME_DT[str(c["x_dtype"])]
    x = dev_tensor(c["x"], xd)
    q, _ = quantize_fp8(x, torch.tensor(float(c["scale"]), device="cuda"), dtype=torch.float8_e4m3fn)
    assert q.dtype == torch.float8_e4m3fn
    got = q.view(torch.uint8).cpu().numpy()
    ref = c["q"]
    nan = (ref & 0x7F) == 0x7F
    np.testing.assert_array_equal(got[~nan], ref[~nan])
    assert ((got[nan] & 0x7F) == 0x7F).all()


def test_e4m3_all_fp16_patterns_vs_torch_cast(cuda):
    from triton_ops import dequantize_fp8, quantize_fp8

    allh = torch.from_numpy(np.arange(65536, dtype=np.uint16).view(np.float16).copy()).cuda()
    finite = torch.isfinite(allh)
    x = allh[finite]
    s = torch.tensor(0.0625, device="cuda")
    q, _ = quantize_fp8(x, s, dtype=torch.float8_e4m3fn)
    ref = (x.float() * s).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(q.view(torch.uint8), ref.view(torch.uint8))
    d = dequantize_fp8(q, s, torch.float32)
    assert torch.equal(d, ref.float() / s)


@pytest.mark.parametrize("amax", [448.0, 200.0, 1.0, 3.7e-3, 65504.0, 1.0e-30])
def test_dynamic_scale_threshold_neighbourhoods(cuda, amax):
    """Dynamic-scale quantize (the in-range fast encode) at every code boundary, bit-exact."""
    from triton_ops import quantize_fp8

    s = O.compute_scale(np.array([amax], np.float32))
    centres = np.array([(k + 0.5) * 448.0 / 127.0 for k in range(-128, 128)], np.float64) / float(s)
    bits = centres.astype(np.float32).view(np.int32)[:, None] + np.arange(-48, 49, dtype=np.int32)[None, :]
    vals = bits.view(np.float32).ravel()
    vals = vals[np.isfinite(vals) & (np.abs(vals) <= np.float32(amax))]
    vals = np.concatenate([np.array([amax, -amax, 0.0, -0.0], np.float32), vals]).astype(np.float32)
    for dt in ("f32", "f16", "bf16"):
        x = O.round_to(vals, dt)
        if not np.isfinite(x).all() or np.abs(x).max() == 0:
            continue
        q, sc = quantize_fp8(dev_tensor(x, dt))
        s_ref = O.compute_scale(x)
        assert f32bits(sc.item()) == f32bits(s_ref)
        np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))


def test_dynamic_scale_all_finite_fp16(cuda):
    """Every finite fp16 value under its own dynamic scale (448 / 65504), both encodings."""
    from triton_ops import quantize_fp8

    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    xh = allh[np.isfinite(allh)].astype(np.float32)
    x = torch.from_numpy(xh.astype(np.float16)).cuda()
    q, s = quantize_fp8(x)
    s_ref = O.compute_scale(xh)
    assert f32bits(s.item()) == f32bits(s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(xh, s_ref))
    q8, s8 = quantize_fp8(x, dtype=torch.float8_e4m3fn)
    ref = (x.float() * s8).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(q8.view(torch.uint8), ref.view(torch.uint8))


def test_dynamic_scale_nan_and_inf_inputs(cuda):
    """amax NaN (scale NaN) and amax inf (scale 0) take the careful encode: codes match the oracle."""
    from triton_ops import quantize_fp8

    rng = np.random.default_rng(3)
    for bad in (np.nan, np.inf, -np.inf):
        x = rng.standard_normal(4099).astype(np.float32)
        x[17] = bad
        q, s = quantize_fp8(torch.from_numpy(x).cuda())
        s_ref = O.compute_scale(x)
        assert f32bits(s.item()) == f32bits(s_ref)
        np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("nvec", [1, 1023, 1024, 1025, 8193, 65535, 65536, 65537])
def test_dynamic_scale_one_cluster_form(cuda, dtype, nvec):
    """Aligned tensors of up to 65536 16-byte vectors take the one-cluster form (one launch, no
    barrier memset; 1-8 CTAs, 2-16 vectors per thread); larger ones the grid-barrier forms. Same
    bytes either way."""
    import torch as _t

    from triton_ops import _lib, quantize_fp8

    ev = 16 // (4 if dtype == "f32" else 2)
    n = nvec * ev
    rng = np.random.default_rng(nvec)
    x = O.round_to((rng.standard_normal(n) * 3).astype(np.float32), dtype)
    xt = dev_tensor(x, dtype)
    for code in (_t.uint8, _t.float8_e4m3fn):
        n0 = _lib.kernel_launches()
        q, s = quantize_fp8(xt, dtype=code)
        launches = _lib.kernel_launches() - n0
        assert (launches == 1) == (nvec <= 65536), launches
        s_ref = O.compute_scale(x)
        assert f32bits(s.item()) == f32bits(s_ref)
        if code == _t.uint8:
            np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))
        else:
            ref = (_t.from_numpy(x.astype(np.float32)) * _t.tensor(s_ref)).clamp(-448, 448).to(_t.float8_e4m3fn)
            assert _t.equal(q.view(_t.uint8).cpu(), ref.view(_t.uint8))
    assert _lib.device_error_flags() == 0


def test_one_cluster_form_nan_inf_and_zero(cuda):
    """The one-cluster form's NaN / inf / all-zero scales and codes equal the oracle's."""
    from triton_ops import quantize_fp8

    rng = np.random.default_rng(4)
    for bad in (np.nan, np.inf, -np.inf, 0.0):
        x = rng.standard_normal(4096).astype(np.float32)
        if bad == 0.0:
            x[:] = 0.0
        else:
            x[17] = bad
        q, s = quantize_fp8(torch.from_numpy(x).cuda())
        s_ref = O.compute_scale(x)
        assert f32bits(s.item()) == f32bits(s_ref)
        np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))


@pytest.mark.parametrize("n,launches", [((8 << 20) - 8, 2), (8 << 20, 2), ((8 << 20) + 8, 2)])
def test_dynamic_scale_partials_and_resident_boundary(cuda, n, launches):
    """fp16 tensors of up to 16 MB use amax partials + encode (two launches); above, the resident form
    (barrier memset + one cooperative launch, also two). Same bytes as the oracle on both sides."""
    from triton_ops import _lib, quantize_fp8

    rng = np.random.default_rng(n % 1000)
    x = O.round_to((rng.standard_normal(n) * 5).astype(np.float32), "f16")
    xt = dev_tensor(x, "f16")
    n0 = _lib.kernel_launches()
    q, s = quantize_fp8(xt)
    assert _lib.kernel_launches() - n0 == launches
    s_ref = O.compute_scale(x)
    assert f32bits(s.item()) == f32bits(s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), O.quantize_ref(x, s_ref))
    assert _lib.device_error_flags() == 0
